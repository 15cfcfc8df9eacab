// k_f32.cu -- f32-activation kernels: dequant_matmul.v1 GEMV, Dequantize and
// embedding rows, with every weight decoded exactly as quant.go does
// (gsoultan/mimir-model quant.go:197-344): Q4_K y = (d*sc)*q - dmin*m,
// Q6_K y = (d*sc)*(q-32), Q8_0 y = d*q, each product rounded on its own.
//
// The v1 GEMV (interp/fast.go:160-224) only has to meet the tolerance of
// spec/stdlib.md section 3.3, so it sums in its own order: one warp owns 4
// weight rows and walks their blocks together, so each activation load
// serves 4 rows; per sub-block it forms sum(x*q) and subtracts the offset
// term once (the factored form of the decode).
#include "common.cuh"
#include "kernels.h"

namespace mimgpu {

namespace {
constexpr unsigned FULL = 0xffffffffu;
constexpr int kRowsPerWarp = 4;
constexpr int kWarps = 8;

struct F32Params {
    GemvSeg seg[kMaxSegs];
    int seg_w0[kMaxSegs + 1];  // first warp-task of each segment
    int nseg;
    const float *x;
    int rows;
    long long K;
};

__device__ __forceinline__ uint32_t ldg_u32(const uint8_t *p) { return __ldg((const unsigned int *)p); }
__device__ __forceinline__ uint32_t ldg_u16(const uint8_t *p) { return __ldg((const unsigned short *)p); }

// Q4_K: lane p covers qs bytes [32c + 4j, +4) of each block, c = p/8,
// j = p%8: 4 low-nibble elements of sub-block 2c and 4 high-nibble ones of 2c+1.
__device__ void v1_q4k(const GemvSeg &sg, int row0, int nrows, const float *x, long long K, float (&acc)[kRowsPerWarp]) {
    const int lane = threadIdx.x & 31, c = lane >> 3, j = lane & 7;
    const long long rb = row_bytes(Q4_K, K);
    const int nb = (int)(K / 256);
    for (int b = 0; b < nb; b++) {
        const float4 xl = __ldg((const float4 *)(x + (long long)b * 256 + 64 * c + 4 * j));
        const float4 xh = __ldg((const float4 *)(x + (long long)b * 256 + 64 * c + 32 + 4 * j));
        const float sl = (xl.x + xl.y) + (xl.z + xl.w), sh = (xh.x + xh.y) + (xh.z + xh.w);
#pragma unroll
        for (int r = 0; r < kRowsPerWarp; r++) {
            if (r >= nrows) break;
            const uint8_t *blk = sg.w + (long long)(row0 + r) * rb + (long long)b * 144;
            const uint4 hdr = __ldg((const uint4 *)blk);
            const uint32_t q = ldg_u32(blk + 16 + 32 * c + 4 * j);
            const uint32_t sw[3] = {hdr.y, hdr.z, hdr.w};
            int sc0, m0, sc1, m1;
            q4k_scale_min(sw, 2 * c, sc0, m0);
            q4k_scale_min(sw, 2 * c + 1, sc1, m1);
            const float d = f16_to_f32(hdr.x & 0xFFFF), dmin = f16_to_f32(hdr.x >> 16);
            const float ql = xl.x * (float)(q & 15) + xl.y * (float)((q >> 8) & 15) + xl.z * (float)((q >> 16) & 15) +
                             xl.w * (float)((q >> 24) & 15);
            const float qhs = xh.x * (float)((q >> 4) & 15) + xh.y * (float)((q >> 12) & 15) +
                              xh.z * (float)((q >> 20) & 15) + xh.w * (float)(q >> 28);
            acc[r] += __fmul_rn(d, (float)sc0) * ql - __fmul_rn(dmin, (float)m0) * sl;
            acc[r] += __fmul_rn(d, (float)sc1) * qhs - __fmul_rn(dmin, (float)m1) * sh;
        }
    }
}

// Q6_K: lane p covers l in {2i, 2i+1} (i = p%16) of half h = p/16: the
// elements 128h + l + {0, 32, 64, 96}.
__device__ void v1_q6k(const GemvSeg &sg, int row0, int nrows, const float *x, long long K, float (&acc)[kRowsPerWarp]) {
    const int lane = threadIdx.x & 31, h = lane >> 4, l = (lane & 15) * 2, is = l >> 4;
    const long long rb = row_bytes(Q6_K, K);
    const int nb = (int)(K / 256);
    for (int b = 0; b < nb; b++) {
        const float *xb = x + (long long)b * 256 + 128 * h + l;
        float2 xv[4];
#pragma unroll
        for (int qq = 0; qq < 4; qq++) xv[qq] = __ldg((const float2 *)(xb + 32 * qq));
#pragma unroll
        for (int r = 0; r < kRowsPerWarp; r++) {
            if (r >= nrows) break;
            const uint8_t *blk = sg.w + (long long)(row0 + r) * rb + (long long)b * 210;
            const uint32_t l0 = ldg_u16(blk + 64 * h + l), l1 = ldg_u16(blk + 64 * h + 32 + l);
            const uint32_t qh = ldg_u16(blk + 128 + 32 * h + l);
            const float d = f16_to_f32(ldg_u16(blk + 208));
            float part = 0.f;
#pragma unroll
            for (int qq = 0; qq < 4; qq++) {
                const uint32_t lw = (qq & 1) ? l1 : l0;
                const int sh = (qq >> 1) * 4;
                const int q0 = (int)(((lw >> sh) & 15) | (((qh >> (2 * qq)) & 3) << 4)) - 32;
                const int q1 = (int)(((lw >> (8 + sh)) & 15) | (((qh >> (8 + 2 * qq)) & 3) << 4)) - 32;
                const int sc = (int)(int8_t)__ldg(blk + 192 + 8 * h + is + 2 * qq);
                part += __fmul_rn(d, (float)sc) * (xv[qq].x * (float)q0 + xv[qq].y * (float)q1);
            }
            acc[r] += part;
        }
    }
}

// Q8_0: lane p takes whole blocks p, p+32, ...
__device__ void v1_q8_0(const GemvSeg &sg, int row0, int nrows, const float *x, long long K, float (&acc)[kRowsPerWarp]) {
    const int lane = threadIdx.x & 31;
    const long long rb = row_bytes(Q8_0, K);
    const int nb = (int)(K / 32);
    for (int b = lane; b < nb; b += 32) {
        float4 xv[8];
#pragma unroll
        for (int i = 0; i < 8; i++) xv[i] = __ldg((const float4 *)(x + (long long)b * 32 + 4 * i));
#pragma unroll
        for (int r = 0; r < kRowsPerWarp; r++) {
            if (r >= nrows) break;
            const uint8_t *blk = sg.w + (long long)(row0 + r) * rb + (long long)b * 34;
            const float d = f16_to_f32(ldg_u16(blk));
            float s = 0.f;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const uint32_t lo = ldg_u16(blk + 2 + 4 * i), hi = ldg_u16(blk + 4 + 4 * i);
                s += xv[i].x * (float)(int8_t)(lo & 0xFF) + xv[i].y * (float)(int8_t)(lo >> 8) +
                     xv[i].z * (float)(int8_t)(hi & 0xFF) + xv[i].w * (float)(int8_t)(hi >> 8);
            }
            acc[r] += d * s;
        }
    }
}

// F16 / F32 weights: lane-strided elements.
__device__ void v1_plain(const GemvSeg &sg, int row0, int nrows, const float *x, long long K, float (&acc)[kRowsPerWarp]) {
    const int lane = threadIdx.x & 31;
    for (long long k = lane; k < K; k += 32) {
        const float xv = __ldg(x + k);
#pragma unroll
        for (int r = 0; r < kRowsPerWarp; r++) {
            if (r >= nrows) break;
            float w;
            if (sg.dt == F16)
                w = f16_to_f32(ldg_u16(sg.w + ((long long)(row0 + r) * K + k) * 2));
            else
                w = __ldg((const float *)sg.w + (long long)(row0 + r) * K + k);
            acc[r] += xv * w;
        }
    }
}

__global__ void __launch_bounds__(kWarps * 32) gemv_f32_kernel(const __grid_constant__ F32Params p) {
    pdl_launch_dependents();
    pdl_wait();
    const int task = blockIdx.x * kWarps + (threadIdx.x >> 5);
    if (task >= p.seg_w0[p.nseg]) return;
    int si = 0;
    while (si + 1 < p.nseg && task >= p.seg_w0[si + 1]) si++;
    const GemvSeg &sg = p.seg[si];
    const int row0 = (task - p.seg_w0[si]) * kRowsPerWarp;
    const int nrows = min(kRowsPerWarp, sg.n - row0);
    for (int a = 0; a < p.rows; a++) {
        const float *x = p.x + (long long)a * p.K;
        float acc[kRowsPerWarp] = {0.f, 0.f, 0.f, 0.f};
        switch (sg.dt) {
        case Q4_K: v1_q4k(sg, row0, nrows, x, p.K, acc); break;
        case Q6_K: v1_q6k(sg, row0, nrows, x, p.K, acc); break;
        case Q8_0: v1_q8_0(sg, row0, nrows, x, p.K, acc); break;
        default: v1_plain(sg, row0, nrows, x, p.K, acc); break;
        }
#pragma unroll
        for (int r = 0; r < kRowsPerWarp; r++) {
            const float s = warp_sum(acc[r]);
            if (r < nrows && (threadIdx.x & 31) == 0) {
                float y = s;
                if (sg.bias) y = __fadd_rn(y, sg.bias[row0 + r]);
                if (sg.res) y = __fadd_rn(sg.res[(long long)a * sg.ldy + row0 + r], y);
                sg.y[(long long)a * sg.ldy + row0 + r] = y;
            }
        }
    }
}

__global__ void dequantize_kernel(int dt, const uint8_t *__restrict__ src, float *__restrict__ dst, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        dst[i] = decode_elem(dt, src, i);
}

// embedding.v1: one row of the table per id; out-of-range ids give zeros.
__global__ void embedding_kernel(int dt, const uint8_t *__restrict__ table, long long V, int E,
                                 const int32_t *__restrict__ ids, float *__restrict__ y, unsigned *epoch) {
    // The first kernel of a forward: its dependents launch only once the
    // previous forward has completed, so they may read what it wrote (the
    // position, the cache rows) before their own grid dependency wait.
    pdl_wait();
    pdl_launch_dependents();
    if (epoch && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *epoch += 1;  // a new forward
    const long long id = ids[blockIdx.x];
    const long long rb = row_bytes(dt, E);
    float *out = y + (long long)blockIdx.x * E;
    const int e = blockIdx.y * blockDim.x + threadIdx.x;  // one element per thread
    if (e < E) out[e] = (id >= 0 && id < V) ? decode_elem(dt, table + id * rb, e) : 0.f;
}

}  // namespace

cudaError_t launch_gemv_f32(const GemvSeg *segs, int nseg, const float *x, int rows, long long K,
                            cudaStream_t st, bool pdl) {
    if (nseg <= 0 || nseg > kMaxSegs) return cudaErrorInvalidValue;
    if (rows <= 0) return cudaSuccess;
    F32Params p = {};
    p.nseg = nseg;
    int t = 0;
    for (int i = 0; i < nseg; i++) {
        if (row_bytes(segs[i].dt, K) == 0 && K != 0) return cudaErrorInvalidValue;
        if ((segs[i].dt == Q4_K || segs[i].dt == Q6_K) && K % 256) return cudaErrorInvalidValue;
        p.seg[i] = segs[i];
        p.seg_w0[i] = t;
        t += (segs[i].n + kRowsPerWarp - 1) / kRowsPerWarp;
    }
    p.seg_w0[nseg] = t;
    if (t == 0) return cudaSuccess;
    p.x = x;
    p.rows = rows;
    p.K = K;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3((t + kWarps - 1) / kWarps);
    cfg.blockDim = dim3(kWarps * 32);
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemv_f32_kernel, p);
}

cudaError_t launch_dequantize(int dt, const uint8_t *src, float *dst, long long n, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    long long blocks = (n + 255) / 256;
    if (blocks > 148LL * 64) blocks = 148LL * 64;
    dequantize_kernel<<<(unsigned)blocks, 256, 0, st>>>(dt, src, dst, n);
    return cudaGetLastError();
}

cudaError_t launch_embedding(int dt, const uint8_t *table, long long V, int E, const int32_t *ids, int n,
                             float *y, cudaStream_t st, bool pdl, unsigned *epoch) {
    if (n <= 0) return cudaSuccess;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3(n, (E + 255) / 256);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, embedding_kernel, dt, table, V, E, ids, y, epoch);
}

}  // namespace mimgpu
