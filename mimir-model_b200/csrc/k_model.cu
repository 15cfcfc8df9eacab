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
#include "p2p.cuh"

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
//
// The block's key rows, then its value rows, stream through a ring of
// shared-memory chunks (kAttnChunk keys of each kv head it reads) filled by
// bulk copies on mbarriers, so every read of the cache is a shared-memory
// read.  A thread computes a whole score: the reference's eight lane
// accumulators a[l] (fma over elements 8c+l) with 16-byte reads.
template <bool F16>
__global__ void __launch_bounds__(256) attn_exact_kernel(AttnArgs2 a) {
    extern __shared__ __align__(128) uint8_t asm_[];
    __shared__ QuantScratch qs;
    __shared__ float red[8][8];
    __shared__ float hsum[8], hmax[8];
    constexpr int ES = F16 ? 2 : 4;
    const int D = a.D, HPB = 256 / D, G = a.H / a.Hkv;
    const int t = blockIdx.y, h0 = blockIdx.x * HPB, tid = threadIdx.x;
    const int nh = min(HPB, a.H - h0);       // heads of this block (fewer in a last partial block)
    const int kv0 = h0 / G, nkv = (h0 + nh - 1) / G - kv0 + 1;
    const size_t rowb = (size_t)D * ES;      // bytes of one key or value row
    const size_t chunkb = (size_t)nkv * kAttnChunk * rowb;
    uint64_t *bar = (uint64_t *)asm_;        // [kAttnRing]
    float *q = (float *)(asm_ + 128);        // [HPB][D]
    float *sc = q + 256;                     // [HPB][C]
    uint8_t *ring = asm_ + (((size_t)128 + sizeof(float) * (256 + (size_t)HPB * a.C) + 127) & ~(size_t)127);
    if (tid == 0) {
        for (int b = 0; b < kAttnRing; b++) mbar_init(&bar[b], 1);
        fence_barrier_init();
    }
    __syncthreads();
    pdl_launch_dependents();
    pdl_wait();
    const int n = (int)(a.pos[t] + 1);
    const int nch = (n + kAttnChunk - 1) / kAttnChunk, items = 2 * nch;  // key chunks, then value chunks
    // item i: chunk i % nch of the keys (i < nch) or the values
    auto issue = [&](int i) {
        const int b = i % kAttnRing, c = i % nch;
        const int j0 = c * kAttnChunk, len = min(kAttnChunk, n - j0);
        const uint8_t *src = (const uint8_t *)(i < nch ? a.kc : a.vc);
        mbar_arrive_expect_tx(&bar[b], (uint32_t)(nkv * len * rowb));
        for (int v = 0; v < nkv; v++)
            bulk_g2s(ring + b * chunkb + v * kAttnChunk * rowb, src + (((size_t)(kv0 + v) * a.C) + j0) * rowb,
                     (uint32_t)(len * rowb), &bar[b]);
    };
    if (tid == 0)
        for (int i = 0; i < min(items, kAttnRing); i++) issue(i);
    if (tid / D < nh) q[tid] = a.qh[((long long)(h0 + tid / D) * a.T + t) * D + tid % D];
    __syncthreads();
    const int n4 = n & ~3;
    bool ok = true;
    // ---- scores, one thread per (key, head) of the chunk
    for (int c = 0; c < nch; c++) {
        const int b = c % kAttnRing, j0 = c * kAttnChunk, len = min(kAttnChunk, n - j0);
        ok &= mbar_wait_bounded(&bar[b], (c / kAttnRing) & 1, a.status);
        for (int it = tid; it < len * nh; it += 256) {
            const int jj = it / nh, hh = it % nh;
            const int kvi = (h0 + hh) / G - kv0;
            const uint8_t *krow = ring + b * chunkb + ((size_t)kvi * kAttnChunk + jj) * rowb;
            const float *qr = q + hh * D;
            float l8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            for (int c8 = 0; c8 < D / 8; c8++) {
                float kv[8];
                if (F16) {
                    const uint4 w = *(const uint4 *)(krow + c8 * 16);
                    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        kv[2 * u] = h2f_bits(ww[u] & 0xFFFFu);
                        kv[2 * u + 1] = h2f_bits(ww[u] >> 16);
                    }
                } else {
                    const float4 w0 = *(const float4 *)(krow + c8 * 32), w1 = *(const float4 *)(krow + c8 * 32 + 16);
                    kv[0] = w0.x; kv[1] = w0.y; kv[2] = w0.z; kv[3] = w0.w;
                    kv[4] = w1.x; kv[5] = w1.y; kv[6] = w1.z; kv[7] = w1.w;
                }
                const float4 q0 = *(const float4 *)(qr + 8 * c8), q1 = *(const float4 *)(qr + 8 * c8 + 4);
                const float qv[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
                for (int l = 0; l < 8; l++) l8[l] = __fmaf_rn(qv[l], kv[l], l8[l]);
            }
            const int j = j0 + jj;
            const float v = j < n4 ? __fadd_rn(__fadd_rn(__fadd_rn(l8[0], l8[1]), __fadd_rn(l8[2], l8[3])),
                                               __fadd_rn(__fadd_rn(l8[4], l8[5]), __fadd_rn(l8[6], l8[7])))
                                   : __fadd_rn(__fadd_rn(__fadd_rn(l8[0], l8[4]), __fadd_rn(l8[1], l8[5])),
                                               __fadd_rn(__fadd_rn(l8[2], l8[6]), __fadd_rn(l8[3], l8[7])));
            sc[hh * a.C + j] = __fmul_rn(v, a.scale);
        }
        __syncthreads();  // every thread is done with buffer b
        if (tid == 0 && c + kAttnRing < items) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(c + kAttnRing);
        }
    }
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
    for (int i = tid; i < n * nh; i += 256) {
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
    // ---- weighted sum of the values: one fused multiply-add per key, in key order
    const int hh = tid / D, d = tid % D;
    const int kvi = (h0 + min(hh, nh - 1)) / G - kv0;
    const float *e = sc + min(hh, nh - 1) * a.C;
    float acc = 0.f;
    for (int c = 0; c < nch; c++) {
        const int i = nch + c, b = i % kAttnRing, j0 = c * kAttnChunk, len = min(kAttnChunk, n - j0);
        ok &= mbar_wait_bounded(&bar[b], (i / kAttnRing) & 1, a.status);
        const uint8_t *vb = ring + b * chunkb + (size_t)kvi * kAttnChunk * rowb + (size_t)d * ES;
#pragma unroll 8
        for (int jj = 0; jj < len; jj++) {
            const float v = F16 ? h2f_bits(*(const uint16_t *)(vb + jj * rowb)) : *(const float *)(vb + jj * rowb);
            acc = __fmaf_rn(e[j0 + jj], v, acc);
        }
        __syncthreads();
        if (tid == 0 && i + kAttnRing < items) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(i + kAttnRing);
        }
    }
    (void)ok;
    if (hh >= nh) return;  // only in a partial block, which never quantizes (E % 256 != 0)
    const float o = __fdiv_rn(acc, hsum[hh]);
    const int E = a.H * D;
    a.out[(long long)t * E + (long long)h0 * D + tid] = o;
    if (a.act.q) quant_block_256(o, t, E, blockIdx.x, a.act, qs);
}

// After the argmax of a greedy step: the picked id (0 when the first logit
// is NaN -- the all-ones key -- or nothing was picked) becomes the next input
// token, is appended to the output ids, the position advances, and the key
// is cleared for the next step.
__global__ void advance_kernel(unsigned long long *key, int32_t *tok, int64_t *pos, int32_t *ids, int *step,
                               P2P wait, const unsigned long long *keys) {
    pdl_wait();
    unsigned long long k = *key;
    if (wait.N > 1) {  // tensor parallelism: this rank's key to every rank, then the largest wins
        for (int r = 0; r < wait.N; r++) peer_ptr<unsigned long long>(wait, r, wait.off)[wait.k] = k;
        p2p_publish_wait(wait);
        k = 0;
        for (int r = 0; r < wait.N; r++) k = max(k, ((volatile const unsigned long long *)keys)[r]);
    }
    const int id = (k == 0 || k == ~0ull) ? 0 : (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
    *key = 0;
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
    const size_t smem = attn_exact_smem(a.H, a.Hkv, a.D, a.C, a.cache_f16);
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

cudaError_t launch_advance(unsigned long long *key, int32_t *tok, int64_t *pos, int32_t *ids, int *step,
                           cudaStream_t st, bool pdl, const P2P *wait, const unsigned long long *keys) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = mk(dim3(1), dim3(1), 0, st, pdl, attr);
    const P2P w = wait ? *wait : P2P{};
    return cudaLaunchKernelEx(&cfg, advance_kernel, key, tok, pos, ids, step, w, keys);
}

}  // namespace mimgpu
