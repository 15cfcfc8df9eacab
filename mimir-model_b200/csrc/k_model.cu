// k_model.cu -- kernels of the device-resident llama step (importer/llama.go:
// 400-534 of gsoultan/mimir-model): RoPE with the key/value cache write,
// split-K attention over the cache, its combine fused with the 8-bit
// quantization of the output, and the greedy-step bookkeeping.
//
// Layouts in HBM: qkv [T, E + 2*Hkv*D] (the three projections side by side),
// q heads [H, T, D], cache [Hkv, C, D] per layer (f16 or f32), attention
// output [T, H*D] (the layout the o projection reads).
#include "common.cuh"
#include "model_kernels.h"
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

__device__ __forceinline__ float h2f(uint32_t h) {  // f16 bits -> f32 (exact)
    float f;
    asm("{ .reg .b16 t; mov.b16 t, %1; cvt.f32.f16 %0, t; }" : "=f"(f) : "h"((unsigned short)h));
    return f;
}

// Split-K attention of the G query heads sharing kv head blockIdx.x, for
// query row blockIdx.y, over the 64 keys [64 s, 64 s + 64) of its visible
// range [0, pos + 1) (the mask j <= p of importer/llama.go:364-397).  The
// key and value rows are staged in shared memory with a 2-word row pad so
// the row-parallel reads below fall on distinct banks.  Writes the split's
// max, sum of exp(s - max) and unnormalised output.
template <bool F16>
__global__ void __launch_bounds__(128) attn_split_kernel(AttnSplitArgs a) {
    extern __shared__ __align__(16) uint32_t sm[];
    const int G = a.H / a.Hkv, D = a.D;
    const int P = (F16 ? D / 2 : D) + 2;      // row pitch in 32-bit words
    float *qs = (float *)sm;                  // [G][D]
    uint32_t *kt = sm + G * D;                // [64][P]
    uint32_t *vt = kt + 64 * P;               // [64][P]
    float *sc = (float *)(vt + 64 * P);       // [G][64]
    float *ml = sc + G * 64;                  // [G][2]
    pdl_launch_dependents();
    pdl_wait();
    const int hk = blockIdx.x, t = blockIdx.y, s = blockIdx.z, tid = threadIdx.x;
    const long long end = a.pos[t] + 1, j0 = (long long)s * 64;
    const long long pidx = ((long long)t * a.H + hk * G) * a.S + s;  // head g adds g*S
    if (j0 >= end) {
        if (tid < G) {
            a.pml[(pidx + (long long)tid * a.S) * 2] = -INFINITY;
            a.pml[(pidx + (long long)tid * a.S) * 2 + 1] = 0.f;
        }
        return;
    }
    const int n = (int)min(64LL, end - j0);
    // stage q, K and V (all loads issued before any use)
    for (int i = tid; i < G * D; i += 128) qs[i] = a.qh[((long long)(hk * G + i / D) * a.T + t) * D + i % D];
    const int wpr = F16 ? D / 2 : D;          // words per key row
    const int cpr = wpr / 4;                  // 16-byte pieces per key row
    const uint4 *kg = (const uint4 *)((const uint32_t *)a.kc + ((long long)hk * a.C + j0) * wpr);
    const uint4 *vg = (const uint4 *)((const uint32_t *)a.vc + ((long long)hk * a.C + j0) * wpr);
    for (int i = tid; i < n * cpr; i += 128) {
        const uint4 k4 = kg[i], v4 = vg[i];
        const int j = i / cpr, c = i % cpr;
        uint32_t *kd = kt + j * P + 4 * c, *vd = vt + j * P + 4 * c;
        *(uint2 *)kd = make_uint2(k4.x, k4.y);
        *(uint2 *)(kd + 2) = make_uint2(k4.z, k4.w);
        *(uint2 *)vd = make_uint2(v4.x, v4.y);
        *(uint2 *)(vd + 2) = make_uint2(v4.z, v4.w);
    }
    __syncthreads();
    // scores: thread (key j, parity hh) dots the words 2i + hh of row j
    {
        const int j = tid >> 1, hh = tid & 1;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if (j < n) {
            const uint32_t *kr = kt + j * P;
            for (int i = 0; i < wpr / 2; i++) {
                const int wi = 2 * i + hh;
                const uint32_t kw = kr[wi];
                if (F16) {
                    const float k0 = h2f(kw & 0xFFFF), k1 = h2f(kw >> 16);
                    for (int g = 0; g < G; g++) {
                        acc[g] = __fmaf_rn(qs[g * D + 2 * wi], k0, acc[g]);
                        acc[g] = __fmaf_rn(qs[g * D + 2 * wi + 1], k1, acc[g]);
                    }
                } else {
                    const float k0 = __uint_as_float(kw);
                    for (int g = 0; g < G; g++) acc[g] = __fmaf_rn(qs[g * D + wi], k0, acc[g]);
                }
            }
        }
        for (int g = 0; g < G; g++) {
            const float v = acc[g] + __shfl_xor_sync(0xffffffffu, acc[g], 1);
            if (hh == 0 && j < n) sc[g * 64 + j] = __fmul_rn(v, a.scale);
        }
    }
    __syncthreads();
    const int lane = tid & 31, w = tid >> 5;
    for (int g = w; g < G; g += 4) {
        float m = -INFINITY;
        for (int j = lane; j < n; j += 32) m = fmaxf(m, sc[g * 64 + j]);
        m = warp_max(m);
        float l = 0.f;
        for (int j = lane; j < n; j += 32) {
            const float e = (float)exp((double)__fsub_rn(sc[g * 64 + j], m));
            sc[g * 64 + j] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) { ml[2 * g] = m; ml[2 * g + 1] = l; }
    }
    __syncthreads();
    for (int d = tid; d < D; d += 128) {
        float o[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int j = 0; j < n; j++) {
            const uint32_t vw = vt[j * P + (F16 ? d >> 1 : d)];
            const float v = F16 ? h2f((d & 1) ? (vw >> 16) : (vw & 0xFFFF)) : __uint_as_float(vw);
            for (int g = 0; g < G; g++) o[g] = __fmaf_rn(sc[g * 64 + j], v, o[g]);
        }
        for (int g = 0; g < G; g++) a.po[(pidx + (long long)g * a.S) * D + d] = o[g];
    }
    if (tid < G) {
        a.pml[(pidx + (long long)tid * a.S) * 2] = ml[2 * tid];
        a.pml[(pidx + (long long)tid * a.S) * 2 + 1] = ml[2 * tid + 1];
    }
}

// Merges the splits of query row blockIdx.x for output elements
// [256 b, 256 b + 256) of out [T, H*D], then quantizes that block (act.q).
__global__ void __launch_bounds__(256) attn_combine_kernel(AttnCombineArgs a) {
    __shared__ QuantScratch qs;
    pdl_launch_dependents();
    pdl_wait();
    const int t = blockIdx.x, b = blockIdx.y, i = b * 256 + threadIdx.x;
    const int E = a.H * a.D;
    const long long end = a.pos[t] + 1;
    const int S = (int)min((long long)a.S, (end + a.chunk - 1) / a.chunk);
    float v = 0.f;
    if (i < E) {
        const int h = i / a.D, d = i % a.D;
        const long long base = ((long long)t * a.H + h) * a.S;
        float M = -INFINITY;
        for (int s = 0; s < S; s++) M = fmaxf(M, a.pml[(base + s) * 2]);
        float L = 0.f, O = 0.f;
        for (int s = 0; s < S; s++) {
            const float f = expf(a.pml[(base + s) * 2] - M);
            L = __fmaf_rn(a.pml[(base + s) * 2 + 1], f, L);
            O = __fmaf_rn(a.po[(base + s) * a.D + d], f, O);
        }
        v = __fdiv_rn(O, L);
        a.out[(long long)t * E + i] = v;
    }
    if (a.act.q) quant_block_256(v, t, E, b, a.act, qs);
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

size_t attn_split_smem(int G, int D, int f16) {
    const int P = (f16 ? D / 2 : D) + 2;
    return sizeof(float) * ((size_t)G * D + 2 * 64 * (size_t)P + (size_t)G * 64 + 2 * G);
}

cudaError_t launch_attn_split(const AttnSplitArgs &a, cudaStream_t st, bool pdl) {
    if (a.T <= 0) return cudaSuccess;
    const int G = a.H / a.Hkv;
    if (G > 8 || a.D % 32 || a.D > 128 || a.chunk != 64) return cudaErrorInvalidValue;
    const size_t smem = attn_split_smem(G, a.D, a.cache_f16);
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = mk(dim3(a.Hkv, a.T, a.S), dim3(128), smem, st, pdl, attr);
    if (a.cache_f16) {
        if (smem > 48 * 1024) {
            cudaError_t e = cudaFuncSetAttribute(attn_split_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
        }
        return cudaLaunchKernelEx(&cfg, attn_split_kernel<true>, a);
    }
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(attn_split_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    return cudaLaunchKernelEx(&cfg, attn_split_kernel<false>, a);
}

cudaError_t launch_attn_combine(const AttnCombineArgs &a, cudaStream_t st, bool pdl) {
    if (a.T <= 0) return cudaSuccess;
    if (a.act.q && (a.H * a.D) % 256) return cudaErrorInvalidValue;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = mk(dim3(a.T, (a.H * a.D + 255) / 256), dim3(256), 0, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, attn_combine_kernel, a);
}

cudaError_t launch_advance(const int *argmax, int32_t *tok, int64_t *pos, int32_t *ids, int *step, cudaStream_t st,
                           bool pdl) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = mk(dim3(1), dim3(1), 0, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, advance_kernel, argmax, tok, pos, ids, step);
}

}  // namespace mimgpu
