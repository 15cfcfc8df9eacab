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

// rope.v1 on the q and k heads of one token (fast.go:507-557), then the cast
// to the cache dtype (RNE f16, prim.go:76-96) and the scatter at the
// token's position (prim.go:278).  One block per token.
__global__ void rope_scatter_kernel(RopeScatterArgs a) {
    extern __shared__ float cs[];
    pdl_launch_dependents();
    pdl_wait();
    const int t = blockIdx.x;
    const int h2 = a.rotary / 2, D = a.D;
    const long long pos = a.pos[t];
    const double pp = (double)pos;
    for (int i = threadIdx.x; i < h2; i += blockDim.x) {
        double s, c;
        sincos(__dmul_rn(pp, a.inv_freq[i]), &s, &c);
        cs[2 * i] = (float)c;
        cs[2 * i + 1] = (float)s;
    }
    __syncthreads();
    const float *row = a.qkv + (long long)t * a.ldq;
    const int nq = a.H * D, nk = a.Hkv * D;
    for (int idx = threadIdx.x; idx < nq + 2 * nk; idx += blockDim.x) {
        float out;
        int head, e;
        const float *src;
        if (idx < nq + nk) {
            const bool isq = idx < nq;
            const int j = isq ? idx : idx - nq;
            head = j / D;
            e = j % D;
            src = row + (isq ? 0 : nq) + head * D;
            if (e >= a.rotary) {
                out = src[e];
            } else {
                int i, first;
                if (a.interleaved) { i = e >> 1; first = !(e & 1); }
                else { i = e < h2 ? e : e - h2; first = e < h2; }
                const int i1 = a.interleaved ? 2 * i : i, i2 = a.interleaved ? 2 * i + 1 : i + h2;
                const float x1 = src[i1], x2 = src[i2], c = cs[2 * i], s = cs[2 * i + 1];
                out = first ? __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s))
                            : __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
            }
            if (isq) {
                a.qh[((long long)head * a.T + t) * D + e] = out;
                continue;
            }
            const long long at = ((long long)head * a.C + pos) * D + e;
            if (a.cache_f16) ((uint16_t *)a.kc)[at] = f32_to_f16(out);
            else ((float *)a.kc)[at] = out;
        } else {
            const int j = idx - nq - nk;
            head = j / D;
            e = j % D;
            out = row[nq + nk + head * D + e];
            const long long at = ((long long)head * a.C + pos) * D + e;
            if (a.cache_f16) ((uint16_t *)a.vc)[at] = f32_to_f16(out);
            else ((float *)a.vc)[at] = out;
        }
    }
}

__device__ __forceinline__ void load_kv(const void *base, int f16, long long off, int n, float *out) {
    if (f16) {
        const uint16_t *p = (const uint16_t *)base + off;
        if (n == 4) {
            const uint2 w = *(const uint2 *)p;
            out[0] = f16_to_f32(w.x & 0xFFFF); out[1] = f16_to_f32(w.x >> 16);
            out[2] = f16_to_f32(w.y & 0xFFFF); out[3] = f16_to_f32(w.y >> 16);
        } else {
            for (int i = 0; i < n; i++) out[i] = f16_to_f32(p[i]);
        }
    } else {
        const float *p = (const float *)base + off;
        for (int i = 0; i < n; i++) out[i] = p[i];
    }
}

// Split-K attention of the G query heads sharing kv head blockIdx.x, for
// query row blockIdx.y, over keys [s*chunk, (s+1)*chunk) of its visible
// range [0, pos+1) (the mask j <= p of importer/llama.go:364-397).  Writes
// the split's max, sum of exp(s - max) and unnormalised output.
__global__ void __launch_bounds__(128) attn_split_kernel(AttnSplitArgs a) {
    extern __shared__ float sm[];
    const int G = a.H / a.Hkv, D = a.D;
    float *qs = sm;                  // [G][D]
    float *sc = sm + G * D;          // [G][chunk]
    float *ml = sc + G * a.chunk;    // [G][2]
    pdl_launch_dependents();
    pdl_wait();
    const int hk = blockIdx.x, t = blockIdx.y, s = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const long long end = a.pos[t] + 1;
    const long long j0 = (long long)s * a.chunk;
    const long long pidx = ((long long)t * a.H + hk * G) * a.S + s;  // head g adds g*S
    if (j0 >= end) {
        if (tid < G) {
            a.pml[(pidx + (long long)tid * a.S) * 2] = -INFINITY;
            a.pml[(pidx + (long long)tid * a.S) * 2 + 1] = 0.f;
        }
        return;
    }
    const int n = (int)min((long long)a.chunk, end - j0);
    for (int i = tid; i < G * D; i += 128) {
        const int g = i / D, d = i % D;
        qs[i] = a.qh[((long long)(hk * G + g) * a.T + t) * D + d];
    }
    __syncthreads();
    const long long kvoff = (long long)hk * a.C * D;
    const int per = D / 32;  // elements per lane (D is a multiple of 32, at most 128)
    for (int j = w; j < n; j += 4) {
        float kv[4];
        load_kv(a.kc, a.cache_f16, kvoff + (j0 + j) * D + lane * per, per, kv);
        for (int g = 0; g < G; g++) {
            float p = 0.f;
            for (int i = 0; i < per; i++) p = __fmaf_rn(qs[g * D + lane * per + i], kv[i], p);
            p = warp_sum(p);
            if (lane == 0) sc[g * a.chunk + j] = __fmul_rn(p, a.scale);
        }
    }
    __syncthreads();
    for (int g = w; g < G; g += 4) {
        float m = -INFINITY;
        for (int j = lane; j < n; j += 32) m = fmaxf(m, sc[g * a.chunk + j]);
        m = warp_max(m);
        float l = 0.f;
        for (int j = lane; j < n; j += 32) {
            const float e = (float)exp((double)__fsub_rn(sc[g * a.chunk + j], m));
            sc[g * a.chunk + j] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) { ml[2 * g] = m; ml[2 * g + 1] = l; }
    }
    __syncthreads();
    for (int d = tid; d < D; d += 128) {
        float o[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int j = 0; j < n; j++) {
            float v;
            load_kv(a.vc, a.cache_f16, kvoff + (j0 + j) * D + d, 1, &v);
            for (int g = 0; g < G; g++) o[g] = __fmaf_rn(sc[g * a.chunk + j], v, o[g]);
        }
        for (int g = 0; g < G; g++) a.po[(pidx + (long long)g * a.S) * D + d] = o[g];
    }
    if (tid < G) {
        a.pml[(pidx + (long long)tid * a.S) * 2] = ml[2 * tid];
        a.pml[(pidx + (long long)tid * a.S) * 2 + 1] = ml[2 * tid + 1];
    }
}

__device__ __forceinline__ void group_sync(int g) { asm volatile("bar.sync %0, 256;" ::"r"(g + 1) : "memory"); }

// Merges the splits of every head of query row blockIdx.x into out [T, H*D],
// then quantizes each 256-element block of the row (act.q non-null).
__global__ void __launch_bounds__(1024) attn_combine_kernel(AttnCombineArgs a) {
    __shared__ float amaxs[4][8];
    __shared__ int bads[4][8];
    pdl_launch_dependents();
    pdl_wait();
    const int t = blockIdx.x, tid = threadIdx.x;
    const int E = a.H * a.D;
    const long long end = a.pos[t] + 1;
    const int S = (int)min((long long)a.S, (end + a.chunk - 1) / a.chunk);
    const int g = tid >> 8, e = tid & 255, w = e >> 5, lane = e & 31;
    bool rowbad = false;
    const int nblk = (E + 255) / 256;
    for (int b = g; b < nblk; b += 4) {
        const int i = b * 256 + e;
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
        if (!a.act.q) continue;
        // 8-bit blocks of the output (q8.go:50-97), as in k_a8.cu
        const float av = fabsf(v);
        const bool bad = !(av <= 0x1p60f);
        const float m = warp_max(bad ? 0.f : av);
        const unsigned anyb = __ballot_sync(0xffffffffu, bad);
        if (lane == 0) { amaxs[g][w] = m; bads[g][w] = anyb != 0; }
        group_sync(g);
        float amax = amaxs[g][0];
        int anybad = bads[g][0];
        for (int k = 1; k < 8; k++) { amax = fmaxf(amax, amaxs[g][k]); anybad |= bads[g][k]; }
        group_sync(g);
        int q = 0;
        if (amax != 0.f && !anybad) q = (int)rint(__ddiv_rn(127.0 * (double)v, (double)amax));
        a.act.q[(long long)t * E + i] = (int8_t)q;
        int s16 = q;
        for (int o = 8; o; o >>= 1) s16 += __shfl_xor_sync(0xffffffffu, s16, o);
        const int s32 = s16 + __shfl_xor_sync(0xffffffffu, s16, 16);
        const long long kb = (long long)t * (E / 256) + b;
        if ((lane & 15) == 0) a.act.ys[kb * 16 + w * 2 + (lane >> 4)] = (int16_t)s16;
        if (lane == 0) a.act.xs[kb * 8 + w] = (int16_t)s32;
        if (e == 0) a.act.dx[kb] = __fdiv_rn(amax, 127.f);
        rowbad |= anybad != 0;
    }
    if (!a.act.q) return;
    const int anybad = __syncthreads_or(rowbad);
    if (tid == 0) a.act.ok[t] = anybad ? 0 : 1;
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
    cudaLaunchConfig_t cfg = mk(dim3(a.T), dim3(256), sizeof(float) * a.rotary, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, rope_scatter_kernel, a);
}

size_t attn_split_smem(int G, int D, int chunk) { return sizeof(float) * ((size_t)G * D + (size_t)G * chunk + 2 * G); }

cudaError_t launch_attn_split(const AttnSplitArgs &a, cudaStream_t st, bool pdl) {
    if (a.T <= 0) return cudaSuccess;
    const int G = a.H / a.Hkv;
    if (G > 8 || a.D % 32 || a.D > 128) return cudaErrorInvalidValue;
    const size_t smem = attn_split_smem(G, a.D, a.chunk);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(attn_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = mk(dim3(a.Hkv, a.T, a.S), dim3(128), smem, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, attn_split_kernel, a);
}

cudaError_t launch_attn_combine(const AttnCombineArgs &a, cudaStream_t st, bool pdl) {
    if (a.T <= 0) return cudaSuccess;
    if (a.act.q && (a.H * a.D) % 256) return cudaErrorInvalidValue;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = mk(dim3(a.T), dim3(1024), 0, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, attn_combine_kernel, a);
}

cudaError_t launch_advance(const int *argmax, int32_t *tok, int64_t *pos, int32_t *ids, int *step, cudaStream_t st,
                           bool pdl) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = mk(dim3(1), dim3(1), 0, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, advance_kernel, argmax, tok, pos, ids, step);
}

}  // namespace mimgpu
