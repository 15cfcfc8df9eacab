// k_a8.cu -- 8-bit activation path of dequant_matmul_a8.v2 (block 256) on sm_100a.
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
// GEMV design: a persistent grid; each CTA owns groups of 8 weight rows.  One
// producer thread streams row slices of up to 16 blocks per row into a
// 4-stage shared-memory ring with cp.async.bulk (the row bytes stay in the
// file's block layout; slices start at the 16-byte boundary below them), and
// 8 consumer warps each take one row: 4 lanes per block, dp4a on the packed
// quants, the block sums reduced with shuffles and folded into the
// block-ordered fma chain.  Activations are read through L1 (they are reused
// by every row).
#include "common.cuh"
#include "kernels.h"

namespace mimgpu {

size_t act_q8_bytes(int rows, long long K) {
    size_t n = 0;
    auto add = [&](size_t b) { n += (b + 255) & ~(size_t)255; };
    add((size_t)rows * K);                      // q
    add((size_t)rows * (K / 256) * 4);          // dx
    add((size_t)rows * (K / 32) * 2);           // xs
    add((size_t)rows * (K / 16) * 2);           // ys
    add((size_t)rows * 4);                      // ok
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
    a.ok = (int *)take((size_t)rows * 4);
    return a;
}

// ------------------------------------------------------------ quantization
//
// The fused kernels run 1024 threads as 4 groups of 256; a group quantizes
// one 256-element activation block at a time and synchronises on its own
// named barrier (ids 1..4), so groups may run different block counts.

__device__ __forceinline__ void group_sync(int g) { asm volatile("bar.sync %0, 256;" ::"r"(g + 1) : "memory"); }

struct QuantScratch {
    float amax[4][8];
    int bad[4][8];
};

// Quantizes one block of 256 activations, v being this thread's element
// (thread t of group g holds element t of the block): amax over the block,
// q = RoundToEven(127*x/amax) in float64, dx = amax/127, and the sums of each
// run of 32 and 16 quants.  Returns whether the block holds a value the
// reference refuses (NaN, Inf, |x| > 2^60).
__device__ __forceinline__ bool quant_block_256(float v, int g, long long row, long long K, int blk, ActQ8 act,
                                                QuantScratch &qs) {
    const int t = threadIdx.x & 255, w = t >> 5, lane = t & 31;
    const float a = fabsf(v);
    const bool bad = !(a <= 0x1p60f);
    const float m = warp_max(bad ? 0.f : a);
    const unsigned anyb = __ballot_sync(0xffffffffu, bad);
    if (lane == 0) {
        qs.amax[g][w] = m;
        qs.bad[g][w] = anyb != 0;
    }
    group_sync(g);
    float amax = qs.amax[g][0];
    int anybad = qs.bad[g][0];
#pragma unroll
    for (int i = 1; i < 8; i++) {
        amax = fmaxf(amax, qs.amax[g][i]);
        anybad |= qs.bad[g][i];
    }
    group_sync(g);  // scratch may be reused by the group's next block
    int q = 0;
    if (amax != 0.f && !anybad) q = (int)rint(__ddiv_rn(127.0 * (double)v, (double)amax));
    act.q[row * K + (long long)blk * 256 + t] = (int8_t)q;
    int s16 = q;
    for (int o = 8; o; o >>= 1) s16 += __shfl_xor_sync(0xffffffffu, s16, o);
    const int s32 = s16 + __shfl_xor_sync(0xffffffffu, s16, 16);
    const long long kb = row * (K / 256) + blk;
    if ((lane & 15) == 0) act.ys[kb * 16 + w * 2 + (lane >> 4)] = (int16_t)s16;
    if (lane == 0) act.xs[kb * 8 + w] = (int16_t)s32;
    if (t == 0) act.dx[kb] = __fdiv_rn(amax, 127.f);
    return anybad != 0;
}

// Writes ok[row] once every group has finished its blocks.
__device__ __forceinline__ void finish_row(bool bad, long long row, ActQ8 act) {
    const int anybad = __syncthreads_or(bad);
    if (threadIdx.x == 0) act.ok[row] = anybad ? 0 : 1;
}

__global__ void __launch_bounds__(1024) quantize_a8_kernel(const float *__restrict__ x, long long K, ActQ8 act) {
    __shared__ QuantScratch qs;
    pdl_launch_dependents();
    pdl_wait();
    const long long row = blockIdx.x;
    const int g = threadIdx.x >> 8, t = threadIdx.x & 255;
    bool bad = false;
    for (int b = g; b < K / 256; b += 4) bad |= quant_block_256(x[row * K + b * 256 + t], g, row, K, b, act, qs);
    finish_row(bad, row, act);
}

// rms_norm (interp/fast.go:434-485) fused with the quantization of its
// output.  The sum of squares is a float64 tree sum (the reference sums in
// order; both round the mean to f32 before the square root).
__global__ void __launch_bounds__(1024) rmsnorm_quant_kernel(const float *__restrict__ x, int n,
                                                             const float *__restrict__ scale, float eps,
                                                             float *__restrict__ y, ActQ8 act) {
    __shared__ double dred[32];
    __shared__ QuantScratch qs;
    pdl_launch_dependents();
    pdl_wait();
    const long long row = blockIdx.x;
    const int t = threadIdx.x;
    const float *xr = x + row * n;
    double ss = 0;
    for (int i = t; i < n; i += 1024) {
        const double e = (double)xr[i];
        ss = __fma_rn(e, e, ss);  // e*e is exact in float64
    }
    ss = warp_sum_d(ss);
    if ((t & 31) == 0) dred[t >> 5] = ss;
    __syncthreads();
    double tot = 0;
#pragma unroll
    for (int i = 0; i < 32; i++) tot += dred[i];
    const float ms = (float)__ddiv_rn(tot, (double)n);
    const float inv = (float)__ddiv_rn(1.0, __dsqrt_rn(__dadd_rn((double)ms, (double)eps)));
    if (!act.q) {
        for (int i = t; i < n; i += 1024) {
            float v = __fmul_rn(xr[i], inv);
            if (scale) v = __fmul_rn(v, scale[i]);
            y[row * n + i] = v;
        }
        return;
    }
    const int g = t >> 8, e = t & 255;
    bool bad = false;
    for (int b = g; b < n / 256; b += 4) {
        const int i = b * 256 + e;
        float v = __fmul_rn(xr[i], inv);
        if (scale) v = __fmul_rn(v, scale[i]);
        y[row * n + i] = v;
        bad |= quant_block_256(v, g, row, n, b, act, qs);
    }
    finish_row(bad, row, act);
}

__device__ __forceinline__ float silu_mul_f64(float a, float b) {
    const double ad = (double)a;
    return (float)__dmul_rn(__ddiv_rn(ad, __dadd_rn(1.0, exp(-ad))), (double)b);
}

// swiglu.v1 (plain-Go SiluMulF32, internal/kernels/attn.go:63-73) fused
// with the quantization of its output for the down projection.
__global__ void __launch_bounds__(1024) swiglu_quant_kernel(const float *__restrict__ gate, const float *__restrict__ up,
                                                            long long ldg, int n, float *__restrict__ y, ActQ8 act) {
    __shared__ QuantScratch qs;
    pdl_launch_dependents();
    pdl_wait();
    const long long row = blockIdx.x;
    const int t = threadIdx.x;
    const float *gr = gate + row * ldg, *ur = up + row * ldg;
    if (!act.q) {
        for (int i = t; i < n; i += 1024) y[row * n + i] = silu_mul_f64(gr[i], ur[i]);
        return;
    }
    const int g = t >> 8, e = t & 255;
    bool bad = false;
    for (int b = g; b < n / 256; b += 4) {
        const int i = b * 256 + e;
        const float v = silu_mul_f64(gr[i], ur[i]);
        y[row * n + i] = v;
        bad |= quant_block_256(v, g, row, n, b, act, qs);
    }
    finish_row(bad, row, act);
}

static cudaLaunchConfig_t rows_cfg(int rows, cudaStream_t st, bool pdl, cudaLaunchAttribute *attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(rows);
    cfg.blockDim = dim3(1024);
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cfg;
}

cudaError_t launch_quantize_a8(const float *x, int rows, long long K, ActQ8 act, cudaStream_t st, bool pdl) {
    if (rows <= 0) return cudaSuccess;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = rows_cfg(rows, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, quantize_a8_kernel, x, K, act);
}

cudaError_t launch_rmsnorm_quant(const float *x, int rows, int n, const float *scale, float eps, float *y,
                                 ActQ8 act, cudaStream_t st, bool pdl) {
    if (rows <= 0) return cudaSuccess;
    if (act.q && n % 256) return cudaErrorInvalidValue;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = rows_cfg(rows, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, rmsnorm_quant_kernel, x, n, scale, eps, y, act);
}

cudaError_t launch_swiglu_quant(const float *gate, const float *up, long long ldg, int rows, int n, float *y,
                                ActQ8 act, cudaStream_t st, bool pdl) {
    if (rows <= 0) return cudaSuccess;
    if (act.q && n % 256) return cudaErrorInvalidValue;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = rows_cfg(rows, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, swiglu_quant_kernel, gate, up, ldg, n, y, act);
}

// ------------------------------------------------------------------ GEMV

namespace {

constexpr int kConsumerWarps = 8;                 // rows per group
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kStages = 4;
constexpr int kKC = 16;                           // blocks of 256 per row slice
constexpr unsigned FULL = 0xffffffffu;

struct A8Params {
    GemvSeg seg[kMaxSegs];
    int seg_g0[kMaxSegs + 1];  // first group of each segment; seg_g0[nseg] = total groups
    int nseg;
    const float *x;
    ActQ8 act;
    int rows;                  // activation rows of this launch (<= NR)
    long long K;
    int nb;                    // K / 256
    int chunks;                // ceil(nb / kKC)
    int slot;                  // bytes per row slot of a stage
    unsigned *status;
};

__device__ __forceinline__ int find_seg(const A8Params &p, int g) {
    int s = 0;
    while (s + 1 < p.nseg && g >= p.seg_g0[s + 1]) s++;
    return s;
}

__device__ __forceinline__ const uint8_t *slice_src(const GemvSeg &s, long long rb, int row, int kb0) {
    return s.w + (long long)row * rb + (long long)kb0 * block_bytes(s.dt);
}

// Exact f32 product of one weight row (decoded as quant.go does) with x,
// for rows the 8-bit path refuses.  Warp-collective; the summation order
// is this kernel's own (the reference's f32 kernels are tolerance-bound).
__device__ float row_dot_f32(int dt, const uint8_t *row, const float *x, int nb) {
    int lane = threadIdx.x & 31;
    float acc = 0.f;
    for (int b = 0; b < nb; b++) {
        const float *xb = x + (long long)b * 256;
        if (dt == Q4_K) {
            const uint8_t *blk = row + (long long)b * 144;
            float d = f16_to_f32(blk[0] | (blk[1] << 8)), dmin = f16_to_f32(blk[2] | (blk[3] << 8));
            uint32_t sw[3];
            for (int i = 0; i < 3; i++)
                sw[i] = blk[4 + 4 * i] | (blk[5 + 4 * i] << 8) | (blk[6 + 4 * i] << 16) | ((uint32_t)blk[7 + 4 * i] << 24);
            for (int e = lane; e < 256; e += 32) {
                int c = e >> 6, hi = (e >> 5) & 1, l = e & 31;
                int sc, m;
                q4k_scale_min(sw, 2 * c + hi, sc, m);
                int qv = hi ? (blk[16 + 32 * c + l] >> 4) : (blk[16 + 32 * c + l] & 15);
                float w = __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)qv), __fmul_rn(dmin, (float)m));
                acc = __fmaf_rn(xb[e], w, acc);
            }
        } else {
            const uint8_t *blk = row + (long long)b * 210;
            float d = f16_to_f32(blk[208] | (blk[209] << 8));
            for (int e = lane; e < 256; e += 32) {
                int h = e >> 7, r = e & 127, quarter = r >> 5, l = r & 31;
                const uint8_t *ql = blk + 64 * h, *qh = blk + 128 + 32 * h;
                int lowb = (quarter & 1) ? ql[l + 32] : ql[l];
                int low = (quarter >> 1) ? (lowb >> 4) : (lowb & 15);
                int high = (qh[l] >> (2 * quarter)) & 3;
                int qv = (low | (high << 4)) - 32;
                int sc = (int8_t)blk[192 + 8 * h + (l >> 4) + 2 * quarter];
                float w = __fmul_rn(__fmul_rn(d, (float)sc), (float)qv);
                acc = __fmaf_rn(xb[e], w, acc);
            }
        }
    }
    return warp_sum(acc);
}

// One slice of a Q4_K row: kbn blocks starting at global block kb0, at
// `slot` in shared memory (16-byte aligned).  Returns true when a block
// scale is not finite.
template <int NR>
__device__ __forceinline__ bool q4k_slice(const uint8_t *slot, int kbn, int kb0, const A8Params &p,
                                          float (&tot)[NR], float (&off)[NR]) {
    const int lane = threadIdx.x & 31, bs = lane >> 2, part = lane & 3;
    bool bad = false;
    for (int pass = 0; pass * 8 < kbn; pass++) {
        const int bl = pass * 8 + bs;
        const bool v = bl < kbn;
        uint4 hdr = make_uint4(0, 0, 0, 0), qa = hdr, qb = hdr;
        if (v) {
            const uint8_t *blk = slot + bl * 144;
            hdr = *(const uint4 *)blk;
            qa = *(const uint4 *)(blk + 16 + 32 * part);
            qb = *(const uint4 *)(blk + 32 + 32 * part);
        }
        const uint32_t dh = hdr.x & 0xFFFFu, mh = hdr.x >> 16;
        bad |= v && (!f16_finite(dh) || !f16_finite(mh));
        const float d = f16_to_f32(dh), dmin = f16_to_f32(mh);
        const uint32_t sw[3] = {hdr.y, hdr.z, hdr.w};
        int sc0, m0, sc1, m1;
        q4k_scale_min(sw, 2 * part, sc0, m0);
        q4k_scale_min(sw, 2 * part + 1, sc1, m1);
        const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        const long long kb = kb0 + bl;
#pragma unroll
        for (int a = 0; a < NR; a++) {
            if (a >= p.rows) break;
            int S = 0, M = 0;
            float dx = 0.f;
            if (v) {
                const int8_t *yq = p.act.q + (long long)a * p.K + kb * 256 + 64 * part;
                const int4 y0 = __ldg((const int4 *)yq), y1 = __ldg((const int4 *)(yq + 16));
                const int4 y2 = __ldg((const int4 *)(yq + 32)), y3 = __ldg((const int4 *)(yq + 48));
                const int ylo[8] = {y0.x, y0.y, y0.z, y0.w, y1.x, y1.y, y1.z, y1.w};
                const int yhi[8] = {y2.x, y2.y, y2.z, y2.w, y3.x, y3.y, y3.z, y3.w};
                int slo = 0, shi = 0;
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    slo = __dp4a((int)(qw[i] & 0x0F0F0F0Fu), ylo[i], slo);
                    shi = __dp4a((int)((qw[i] >> 4) & 0x0F0F0F0Fu), yhi[i], shi);
                }
                S = sc0 * slo + sc1 * shi;
                const int xw = __ldg((const int *)(p.act.xs + (long long)a * (p.K / 32) + kb * 8 + 2 * part));
                M = m0 * (int)(int16_t)(xw & 0xFFFF) + m1 * (int)(int16_t)((unsigned)xw >> 16);
                dx = __ldg(p.act.dx + (long long)a * p.nb + kb);
            }
            S += __shfl_xor_sync(FULL, S, 1);
            S += __shfl_xor_sync(FULL, S, 2);
            M += __shfl_xor_sync(FULL, M, 1);
            M += __shfl_xor_sync(FULL, M, 2);
            const float fs = __int2float_rn(S), pd = __fmul_rn(d, dx);
            const float fm = __int2float_rn(M), pm = __fmul_rn(dmin, dx);
#pragma unroll
            for (int b = 0; b < 8; b++) {
                const float a1 = __shfl_sync(FULL, fs, 4 * b), a2 = __shfl_sync(FULL, pd, 4 * b);
                const float a3 = __shfl_sync(FULL, fm, 4 * b), a4 = __shfl_sync(FULL, pm, 4 * b);
                if (pass * 8 + b < kbn) {
                    tot[a] = __fmaf_rn(a1, a2, tot[a]);
                    off[a] = __fmaf_rn(a3, a4, off[a]);
                }
            }
        }
    }
    return __any_sync(FULL, bad);
}

// One slice of a Q6_K row.  Blocks are 210 bytes, so block starts are only
// 2-byte aligned; words are read from shared memory and realigned.
template <int NR>
__device__ __forceinline__ bool q6k_slice(const uint8_t *slot, int kbn, int kb0, const A8Params &p,
                                          float (&tot)[NR]) {
    const int lane = threadIdx.x & 31, bs = lane >> 2, part = lane & 3;
    const int h = part >> 1, lq = (part & 1) * 16;
    bool bad = false;
    for (int pass = 0; pass * 8 < kbn; pass++) {
        const int bl = pass * 8 + bs;
        const bool v = bl < kbn;
        uint32_t l0[4] = {0, 0, 0, 0}, l1[4] = {0, 0, 0, 0}, qh[4] = {0, 0, 0, 0};
        uint32_t scw0 = 0, scw1 = 0, dh = 0;
        if (v) {
            const uint8_t *blk = slot + bl * 210;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                l0[i] = lds_u32_unaligned(blk + 64 * h + lq + 4 * i);
                l1[i] = lds_u32_unaligned(blk + 64 * h + 32 + lq + 4 * i);
                qh[i] = lds_u32_unaligned(blk + 128 + 32 * h + lq + 4 * i);
            }
            scw0 = lds_u32_unaligned(blk + 192 + 8 * h + (lq >> 4));
            scw1 = lds_u32_unaligned(blk + 196 + 8 * h + (lq >> 4));
            dh = lds_u32_unaligned(blk + 208) & 0xFFFFu;
        }
        bad |= v && !f16_finite(dh);
        const float d = f16_to_f32(dh);
        const int sc0 = (int)(int8_t)(scw0 & 0xFF), sc2 = (int)(int8_t)((scw0 >> 16) & 0xFF);
        const int sc4 = (int)(int8_t)(scw1 & 0xFF), sc6 = (int)(int8_t)((scw1 >> 16) & 0xFF);
        uint32_t Q1[4], Q2[4], Q3[4], Q4[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            Q1[i] = (l0[i] & 0x0F0F0F0Fu) | ((qh[i] & 0x03030303u) << 4);
            Q2[i] = (l1[i] & 0x0F0F0F0Fu) | (((qh[i] >> 2) & 0x03030303u) << 4);
            Q3[i] = ((l0[i] >> 4) & 0x0F0F0F0Fu) | (((qh[i] >> 4) & 0x03030303u) << 4);
            Q4[i] = ((l1[i] >> 4) & 0x0F0F0F0Fu) | (((qh[i] >> 6) & 0x03030303u) << 4);
        }
        const long long kb = kb0 + bl;
        const long long e0 = kb * 256 + 128 * h + lq;
#pragma unroll
        for (int a = 0; a < NR; a++) {
            if (a >= p.rows) break;
            int S = 0;
            float dx = 0.f;
            if (v) {
                const int8_t *yq = p.act.q + (long long)a * p.K + e0;
                const int4 y1 = __ldg((const int4 *)yq), y2 = __ldg((const int4 *)(yq + 32));
                const int4 y3 = __ldg((const int4 *)(yq + 64)), y4 = __ldg((const int4 *)(yq + 96));
                int s1 = 0, s2 = 0, s3 = 0, s4 = 0;
                s1 = __dp4a((int)Q1[0], y1.x, s1); s1 = __dp4a((int)Q1[1], y1.y, s1);
                s1 = __dp4a((int)Q1[2], y1.z, s1); s1 = __dp4a((int)Q1[3], y1.w, s1);
                s2 = __dp4a((int)Q2[0], y2.x, s2); s2 = __dp4a((int)Q2[1], y2.y, s2);
                s2 = __dp4a((int)Q2[2], y2.z, s2); s2 = __dp4a((int)Q2[3], y2.w, s2);
                s3 = __dp4a((int)Q3[0], y3.x, s3); s3 = __dp4a((int)Q3[1], y3.y, s3);
                s3 = __dp4a((int)Q3[2], y3.z, s3); s3 = __dp4a((int)Q3[3], y3.w, s3);
                s4 = __dp4a((int)Q4[0], y4.x, s4); s4 = __dp4a((int)Q4[1], y4.y, s4);
                s4 = __dp4a((int)Q4[2], y4.z, s4); s4 = __dp4a((int)Q4[3], y4.w, s4);
                const int16_t *ys = p.act.ys + (long long)a * (p.K / 16) + e0 / 16;
                S = sc0 * (s1 - 32 * (int)__ldg(ys)) + sc2 * (s2 - 32 * (int)__ldg(ys + 2)) +
                    sc4 * (s3 - 32 * (int)__ldg(ys + 4)) + sc6 * (s4 - 32 * (int)__ldg(ys + 6));
                dx = __ldg(p.act.dx + (long long)a * p.nb + kb);
            }
            S += __shfl_xor_sync(FULL, S, 1);
            S += __shfl_xor_sync(FULL, S, 2);
            const float fs = __int2float_rn(S), pd = __fmul_rn(d, dx);
#pragma unroll
            for (int b = 0; b < 8; b++) {
                const float a1 = __shfl_sync(FULL, fs, 4 * b), a2 = __shfl_sync(FULL, pd, 4 * b);
                if (pass * 8 + b < kbn) tot[a] = __fmaf_rn(a1, a2, tot[a]);
            }
        }
    }
    return __any_sync(FULL, bad);
}

template <int NR>
__global__ void __launch_bounds__(kThreads) gemv_a8_kernel(const __grid_constant__ A8Params p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = (uint64_t *)smem;
    uint64_t *empty = full + kStages;
    uint8_t *tiles = smem + 128;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int total_groups = p.seg_g0[p.nseg];

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        fence_barrier_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == kConsumerWarps) {
        // ---------------- producer: weights do not depend on the previous
        // kernel, so they stream in before the activations are ready.
        if (lane != 0) return;
        int it = 0;
        bool ok = true;
        for (int g = blockIdx.x; g < total_groups && ok; g += gridDim.x) {
            const int si = find_seg(p, g);
            const GemvSeg &sg = p.seg[si];
            const long long rb = row_bytes(sg.dt, p.K);
            const int r0 = (g - p.seg_g0[si]) * kConsumerWarps;
            const int nrows = min(kConsumerWarps, sg.n - r0);
            const int bb = block_bytes(sg.dt);
            for (int c = 0; c < p.chunks && ok; c++, it++) {
                const int s = it % kStages;
                if (it >= kStages) ok = mbar_wait_bounded(&empty[s], ((it / kStages) - 1) & 1, p.status);
                if (!ok) break;
                const int kb0 = c * kKC, kbn = min(kKC, p.nb - kb0);
                uint32_t total = 0;
                for (int r = 0; r < nrows; r++) {
                    uintptr_t a = (uintptr_t)slice_src(sg, rb, r0 + r, kb0);
                    uintptr_t lo = a & ~(uintptr_t)15, hi = (a + (uintptr_t)kbn * bb + 15) & ~(uintptr_t)15;
                    total += (uint32_t)(hi - lo);
                }
                mbar_arrive_expect_tx(&full[s], total);
                for (int r = 0; r < nrows; r++) {
                    uintptr_t a = (uintptr_t)slice_src(sg, rb, r0 + r, kb0);
                    uintptr_t lo = a & ~(uintptr_t)15, hi = (a + (uintptr_t)kbn * bb + 15) & ~(uintptr_t)15;
                    bulk_g2s(tiles + ((size_t)s * kConsumerWarps + r) * p.slot, (const void *)lo,
                             (uint32_t)(hi - lo), &full[s]);
                }
            }
        }
        // Wait (bounded) for the copies still in flight before leaving, so
        // that none lands in shared memory after the block has exited.
        for (int u = max(0, it - kStages); u < it; u++) mbar_wait_bounded(&full[u % kStages], (u / kStages) & 1, p.status);
        return;
    }

    // -------------------- consumers: warp w owns row w of each group
    pdl_wait();
    int it = 0;
    for (int g = blockIdx.x; g < total_groups; g += gridDim.x) {
        const int si = find_seg(p, g);
        const GemvSeg &sg = p.seg[si];
        const long long rb = row_bytes(sg.dt, p.K);
        const int row = (g - p.seg_g0[si]) * kConsumerWarps + warp;
        const bool valid = row < sg.n;
        float tot[NR], off[NR];
#pragma unroll
        for (int a = 0; a < NR; a++) tot[a] = off[a] = 0.f;
        bool refused = false;
        for (int c = 0; c < p.chunks; c++, it++) {
            const int s = it % kStages;
            if (!mbar_wait_bounded(&full[s], (it / kStages) & 1, p.status)) return;
            const int kb0 = c * kKC, kbn = min(kKC, p.nb - kb0);
            if (valid && !refused) {
                const uint8_t *src = slice_src(sg, rb, row, kb0);
                const uint8_t *slot = tiles + ((size_t)s * kConsumerWarps + warp) * p.slot + ((uintptr_t)src & 15);
                if (sg.dt == Q4_K)
                    refused = q4k_slice<NR>(slot, kbn, kb0, p, tot, off);
                else
                    refused = q6k_slice<NR>(slot, kbn, kb0, p, tot);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        if (!valid) continue;
#pragma unroll
        for (int a = 0; a < NR; a++) {
            if (a >= p.rows) break;
            float r;
            if (!refused && p.act.ok[a])
                r = __fsub_rn(tot[a], off[a]);
            else
                r = row_dot_f32(sg.dt, sg.w + (long long)row * rb, p.x + (long long)a * p.K, p.nb);
            if (sg.bias) r = __fadd_rn(r, sg.bias[row]);
            if (sg.res) r = __fadd_rn(sg.res[(long long)a * sg.ldy + row], r);
            if (lane == 0) sg.y[(long long)a * sg.ldy + row] = r;
        }
    }
}

constexpr size_t kMaxSmem = 128 + (size_t)kStages * kConsumerWarps * ((kKC * 210 + 32 + 15) & ~15);

template <int NR>
cudaError_t prepare_nr() {
    static bool done = false;
    if (done) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(gemv_a8_kernel<NR>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxSmem);
    if (e == cudaSuccess) done = true;
    return e;
}

template <int NR>
int blocks_per_sm(size_t smem) {
    static size_t key[4] = {0, 0, 0, 0};
    static int val[4] = {0, 0, 0, 0};
    for (int i = 0; i < 4; i++)
        if (key[i] == smem) return val[i];
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_a8_kernel<NR>, kThreads, smem) != cudaSuccess)
        per_sm = 1;
    for (int i = 0; i < 4; i++)
        if (key[i] == 0) {
            key[i] = smem;
            val[i] = per_sm;
            break;
        }
    return per_sm;
}

template <int NR>
cudaError_t launch_nr(A8Params &p, cudaStream_t st, bool pdl) {
    const size_t smem = 128 + (size_t)kStages * kConsumerWarps * p.slot;
    cudaError_t e = prepare_nr<NR>();
    if (e != cudaSuccess) return e;
    const int per_sm = max(1, blocks_per_sm<NR>(smem));
    const int total = p.seg_g0[p.nseg];
    const int grid = min(total, per_sm * num_sms());
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemv_a8_kernel<NR>, p);
}

}  // namespace

cudaError_t gemv_a8_prepare() {
    cudaError_t e = prepare_nr<1>();
    if (e == cudaSuccess) e = prepare_nr<2>();
    if (e == cudaSuccess) e = prepare_nr<4>();
    if (e == cudaSuccess) e = prepare_nr<8>();
    num_sms();
    return e;
}

cudaError_t launch_gemv_a8(const GemvSeg *segs, int nseg, const float *x, ActQ8 act, int rows, long long K,
                           unsigned *status, cudaStream_t st, bool pdl) {
    if (nseg <= 0 || nseg > kMaxSegs || K % 256 != 0 || rows < 0) return cudaErrorInvalidValue;
    if (rows == 0 || K == 0) return cudaSuccess;
    A8Params p = {};
    p.nseg = nseg;
    int maxbb = 0, g = 0;
    for (int i = 0; i < nseg; i++) {
        if (segs[i].dt != Q4_K && segs[i].dt != Q6_K) return cudaErrorInvalidValue;
        p.seg[i] = segs[i];
        p.seg_g0[i] = g;
        g += (segs[i].n + kConsumerWarps - 1) / kConsumerWarps;
        maxbb = max(maxbb, block_bytes(segs[i].dt));
    }
    p.seg_g0[nseg] = g;
    if (g == 0) return cudaSuccess;
    p.K = K;
    p.nb = (int)(K / 256);
    p.chunks = (p.nb + kKC - 1) / kKC;
    p.slot = (min(kKC, p.nb) * maxbb + 32 + 15) & ~15;
    p.status = status;
    cudaError_t e = cudaSuccess;
    // activation rows go through in launches of at most 8
    for (int r0 = 0; r0 < rows && e == cudaSuccess; r0 += 8) {
        const int nr = min(8, rows - r0);
        A8Params q = p;
        q.rows = nr;
        q.x = x + (long long)r0 * K;
        q.act.q = act.q + (long long)r0 * K;
        q.act.dx = act.dx + (long long)r0 * (K / 256);
        q.act.xs = act.xs + (long long)r0 * (K / 32);
        q.act.ys = act.ys + (long long)r0 * (K / 16);
        q.act.ok = act.ok + r0;
        for (int i = 0; i < nseg; i++) {
            q.seg[i].y = segs[i].y + (long long)r0 * segs[i].ldy;
            if (segs[i].res) q.seg[i].res = segs[i].res + (long long)r0 * segs[i].ldy;
        }
        if (nr == 1)
            e = launch_nr<1>(q, st, pdl);
        else if (nr == 2)
            e = launch_nr<2>(q, st, pdl);
        else if (nr <= 4)
            e = launch_nr<4>(q, st, pdl);
        else
            e = launch_nr<8>(q, st, pdl);
    }
    return e;
}

}  // namespace mimgpu
