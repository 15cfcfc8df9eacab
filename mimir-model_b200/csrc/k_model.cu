// k_model.cu -- kernels of the device-resident llama step (importer/llama.go:
// 400-534 of gsoultan/mimir-model): RoPE with the key/value cache write,
// attention over the cache with the reference's amd64 arithmetic fused with
// the 8-bit quantization of its output, and the greedy-step bookkeeping.
//
// Layouts in HBM: qkv [T, E + 2*Hkv*D] (the three projections side by side),
// q heads [H, T, D], cache [Hkv, C, D] per layer (f16 or f32), attention
// output [T, H*D] (the layout the o projection reads).
#include "common.cuh"
#include "model_kernels.h"
#include "amd64_math.cuh"
#include "quant.cuh"

namespace mimgpu {

namespace {

cudaLaunchConfig_t mk(dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl, cudaLaunchAttribute *attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cfg;
}

// rope.v1 (fast.go:507-557) on one head of one token per block
// (blockIdx.y < H: a query head; < H + Hkv: a key head, cast to the cache
// dtype (RNE f16, prim.go:76-96) and scattered at the token's position
// (prim.go:278); otherwise a value head, cast and scattered).
__global__ void rope_scatter_kernel(RopeScatterArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    const int t = blockIdx.x, hi = blockIdx.y, e = threadIdx.x, D = a.D;
    if (e >= D) return;
    const long long pos = a.pos[t];
    const float *row = a.qkv + (long long)t * a.ldq;
    const int nq = a.H * D, nk = a.Hkv * D;
    if (hi >= a.H + a.Hkv) {  // value head
        const int head = hi - a.H - a.Hkv;
        const float v = row[nq + nk + head * D + e];
        const long long at = ((long long)head * a.C + pos) * D + e;
        if (a.cache_f16) ((uint16_t *)a.vc)[at] = f32_to_f16(v);
        else ((float *)a.vc)[at] = v;
        return;
    }
    const bool isq = hi < a.H;
    const int head = isq ? hi : hi - a.H;
    const float *src = row + (isq ? 0 : nq) + head * D;
    float out;
    const int h2 = a.rotary / 2;
    if (e >= a.rotary) {
        out = src[e];
    } else {
        int i, first;
        if (a.interleaved) { i = e >> 1; first = !(e & 1); }
        else { i = e < h2 ? e : e - h2; first = e < h2; }
        const int i1 = a.interleaved ? 2 * i : i, i2 = a.interleaved ? 2 * i + 1 : i + h2;
        double sd, cd;
        sincos(__dmul_rn((double)pos, a.inv_freq[i]), &sd, &cd);
        const float c = (float)cd, s = (float)sd, x1 = src[i1], x2 = src[i2];
        out = first ? __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s)) : __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
    }
    if (isq) {
        a.qh[((long long)head * a.T + t) * D + e] = out;
        return;
    }
    const long long at = ((long long)head * a.C + pos) * D + e;
    if (a.cache_f16) ((uint16_t *)a.kc)[at] = f32_to_f16(out);
    else ((float *)a.kc)[at] = out;
}

// attention.v2 (attention.v1 for an f32 cache) of HPB = 256/D query heads
// h0 = HPB*blockIdx.x.. of query row t = blockIdx.y over the keys [0, pos+1)
// its mask admits (j <= p, importer/llama.go:364-397), computed exactly as
// attendRow (interp/fast.go:728-751) with the reference's amd64 kernels:
// scores as scoresF16AVX2 (8 fused lanes, group-of-four / tail orders),
// ExpSumF32 (Cephes expf on the first n&~7 keys with its lane-sum order,
// float64 exp on the rest), the fused key-ordered weighted sum of wsumF16AVX2,
// o = acc/sum.  The 256 outputs of the block (H*D row-major, the layout the o
// projection reads) are then quantized to 8 bits when act.q is set.
template <bool F16>
__global__ void __launch_bounds__(256) attn_exact_kernel(AttnArgs2 a) {
    extern __shared__ float asmem[];
    __shared__ QuantScratch qs;
    __shared__ float red[8][8];
    __shared__ float hsum[8], hmax[8];
    pdl_launch_dependents();
    pdl_wait();
    const int D = a.D, HPB = 256 / D, G = a.H / a.Hkv;
    const int t = blockIdx.y, h0 = blockIdx.x * HPB, tid = threadIdx.x;
    const int nh = min(HPB, a.H - h0);  // heads of this block (fewer in a last partial block)
    const int n = (int)(a.pos[t] + 1);
    float *q = asmem;                   // [HPB][D]
    float *sc = asmem + 256;            // [HPB][C]
    if (tid / D < nh) q[tid] = a.qh[((long long)(h0 + tid / D) * a.T + t) * D + tid % D];
    __syncthreads();
    // scores: an 8-lane group per (key, head); group g of pass u takes item
    // base + 32 u + g: key item / nh, head item % nh
    const int l = tid & 7, grp = tid >> 3;
    const int n4 = n & ~3, items = n * nh;
    for (int base = 0; base < items; base += 32 * 4) {
        float acc[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int item = base + 32 * u + grp;
            acc[u] = 0.f;
            if (item < items) {
                const int j = item / nh, hh = item % nh;
                const long long kr = ((long long)((h0 + hh) / G) * a.C + j) * D;
                const float *qr = q + hh * D;
                for (int c = 0; c < D / 8; c++) {
                    const float kv = F16 ? h2f_bits(((const uint16_t *)a.kc)[kr + 8 * c + l])
                                         : ((const float *)a.kc)[kr + 8 * c + l];
                    acc[u] = __fmaf_rn(qr[8 * c + l], kv, acc[u]);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int item = base + 32 * u + grp;
            const int j = item / nh;
            const float v = score_combine(acc[u], j >= n4);  // the 8 lanes of a group share j
            if (item < items && l == 0) sc[(item % nh) * a.C + j] = __fmul_rn(v, a.scale);
        }
    }
    __syncthreads();
    // max per head (warp hh); exact in any order
    const int lane = tid & 31, w = tid >> 5;
    if (w < nh) {
        float m = -INFINITY;
        for (int j = lane; j < n; j += 32) m = fmaxf(m, sc[w * a.C + j]);
        m = warp_max(m);
        if (lane == 0) hmax[w] = m;
    }
    __syncthreads();
    // exp of the scores: Cephes on the first n&~7 keys (none when n < 8)
    const int n8 = n >= 8 ? (n & ~7) : 0;
    for (int i = tid; i < items; i += 256) {
        const int hh = i / n, j = i % n;
        const float x = __fsub_rn(sc[hh * a.C + j], hmax[hh]);
        sc[hh * a.C + j] = j < n8 ? expf_amd64(x) : (float)exp((double)x);
    }
    __syncthreads();
    // ExpSumF32's sum: 8 lane sums in key order, combined, then the tail in order
    if (tid < 8 * nh) {
        const int hh = tid >> 3, ll = tid & 7;
        float sl = 0.f;
        for (int j = ll; j < n8; j += 8) sl = __fadd_rn(sl, sc[hh * a.C + j]);
        red[hh][ll] = sl;
    }
    __syncthreads();
    if (tid < nh) {
        const float *r = red[tid];
        float sum = 0.f;
        if (n8) sum = __fadd_rn(__fadd_rn(__fadd_rn(r[0], r[4]), __fadd_rn(r[1], r[5])),
                                __fadd_rn(__fadd_rn(r[2], r[6]), __fadd_rn(r[3], r[7])));
        for (int j = n8; j < n; j++) sum = __fadd_rn(sum, sc[tid * a.C + j]);
        hsum[tid] = sum;
    }
    __syncthreads();
    // weighted sum of the values: one fused multiply-add per key, in key order
    const int hh = tid / D, d = tid % D;
    if (hh >= nh) return;  // only in a partial block, which never quantizes (E % 256 != 0)
    const long long vr = (long long)((h0 + hh) / G) * a.C * D + d;
    const float *e = sc + hh * a.C;
    float acc = 0.f;
    int j = 0;
    for (; j + 8 <= n; j += 8) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; u++)
            v[u] = F16 ? h2f_bits(((const uint16_t *)a.vc)[vr + (long long)(j + u) * D])
                       : ((const float *)a.vc)[vr + (long long)(j + u) * D];
#pragma unroll
        for (int u = 0; u < 8; u++) acc = __fmaf_rn(e[j + u], v[u], acc);
    }
    for (; j < n; j++) {
        const float v = F16 ? h2f_bits(((const uint16_t *)a.vc)[vr + (long long)j * D])
                            : ((const float *)a.vc)[vr + (long long)j * D];
        acc = __fmaf_rn(e[j], v, acc);
    }
    const float o = __fdiv_rn(acc, hsum[hh]);
    const int E = a.H * D;
    a.out[(long long)t * E + (long long)h0 * D + tid] = o;
    if (a.act.q) quant_block_256(o, t, E, blockIdx.x, a.act, qs);
}

// After the argmax of a greedy step: the picked id becomes the next input
// token, is appended to the output ids, and the position advances.
__global__ void advance_kernel(const int *argmax, int32_t *tok, int64_t *pos, int32_t *ids, int *step) {
    pdl_wait();
    const int id = *argmax;
    *tok = id;
    ids[*step] = id;
    *step += 1;
    *pos += 1;
}

}  // namespace

cudaError_t launch_rope_scatter(const RopeScatterArgs &a, cudaStream_t st, bool pdl) {
    if (a.T <= 0) return cudaSuccess;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = mk(dim3(a.T, a.H + 2 * a.Hkv), dim3((a.D + 31) / 32 * 32), 0, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, rope_scatter_kernel, a);
}

cudaError_t launch_attn_exact(const AttnArgs2 &a, cudaStream_t st, bool pdl) {
    if (a.T <= 0) return cudaSuccess;
    // heads of 32..256 elements dividing 256; the fused quantization needs
    // whole blocks of 256 outputs
    if (a.D < 32 || 256 % a.D || a.Hkv <= 0 || a.H % a.Hkv || (a.act.q && a.H % (256 / a.D)))
        return cudaErrorInvalidValue;
    const int HPB = 256 / a.D;
    const size_t smem = attn_exact_smem(a.D, a.C);
    if (smem > kAttnSmemMax) return cudaErrorInvalidValue;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = mk(dim3((a.H + HPB - 1) / HPB, a.T), dim3(256), smem, st, pdl, attr);
    if (a.cache_f16) {
        cudaError_t e = cudaFuncSetAttribute(attn_exact_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        return cudaLaunchKernelEx(&cfg, attn_exact_kernel<true>, a);
    }
    cudaError_t e = cudaFuncSetAttribute(attn_exact_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    return cudaLaunchKernelEx(&cfg, attn_exact_kernel<false>, a);
}

cudaError_t launch_advance(const int *argmax, int32_t *tok, int64_t *pos, int32_t *ids, int *step, cudaStream_t st,
                           bool pdl) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = mk(dim3(1), dim3(1), 0, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, advance_kernel, argmax, tok, pos, ids, step);
}

}  // namespace mimgpu
