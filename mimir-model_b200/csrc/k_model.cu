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
        const long long at = (a.slot ? a.slot[t] : a.slot0) * cache_slot_elems(a.Hkv, a.C, D) +
                             ((long long)head * a.C + pos) * D + e;
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
        float c, s;
        if (a.rope_cs) {  // the session's table: the same float64 sincos, rounded
            const float2 cs = a.rope_cs[pos * h2 + i];
            c = cs.x;
            s = cs.y;
        } else {
            double sd, cd;
            sincos(__dmul_rn((double)pos, a.inv_freq[i]), &sd, &cd);
            c = (float)cd;
            s = (float)sd;
        }
        const float x1 = src[i1], x2 = src[i2];
        out = first ? __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s)) : __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
    }
    if (isq) {
        a.qh[((long long)head * a.T + t) * D + e] = out;
        return;
    }
    const long long at = (a.slot ? a.slot[t] : a.slot0) * cache_slot_elems(a.Hkv, a.C, D) +
                         ((long long)head * a.C + pos) * D + e;
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
    const size_t slot_off = (size_t)(a.slot ? a.slot[t] : a.slot0) * cache_slot_elems(a.Hkv, a.C, D) * ES;
    auto issue = [&](int i) {
        const int b = i % kAttnRing, c = i % nch;
        const int j0 = c * kAttnChunk, len = min(kAttnChunk, n - j0);
        const uint8_t *src = (const uint8_t *)(i < nch ? a.kc : a.vc) + slot_off;
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
    const int E = a.H * D;
    float o = 0.f;
    if (hh < nh) {
        o = __fdiv_rn(acc, hsum[hh]);
        a.out[(long long)t * E + (long long)h0 * D + tid] = o;
        // tensor parallelism: this rank's heads into every rank's full vector
        for (int r = 0; r < (a.put.N > 1 ? a.put.N : 0); r++)
            peer_ptr<float>(a.put, r, a.put.off)[a.put.col0 + (long long)h0 * D + tid] = o;
    }
    if (a.put.N > 1) {
        // the block's peer stores are visible system-wide before the kernel
        // ends (the next kernel on this stream publishes the exchange)
        __syncthreads();
        if (tid == 0) __threadfence_system();
    }
    if (hh >= nh) return;  // only in a partial block, which never quantizes (E % 256 != 0)
    if (a.act.q) quant_block_256(o, t, E, blockIdx.x, a.act, qs);
}

// attention.v2 for many query rows at once (a prompt pass), f16 cache, D = 128:
// the same arithmetic as attn_exact_kernel row by row -- scores in the eight-
// lane orders, Cephes expf on the first n&~7 keys of the row, ExpSumF32's
// lane-sum order, the key-ordered fused weighted sum, o = acc/sum -- so every
// row's output has the bits the one-row kernel gives it.  A block takes one kv
// head and PQ query rows x its G heads (32 rows), so each key and value row
// read from the cache serves 32 rows instead of one.  Two passes: the first
// computes the scores into a global scratch (L2-resident for short prompts)
// and each row's maximum, the second reads them back, exponentiates, sums
// and accumulates the values.  Keys, then values, stream through a ring of
// 32-row chunks (bulk copies on mbarriers), widened to f32 once per chunk in
// shared memory.  Register tiles: a lane
// scores 4 rows against 1 key (rows and keys in rows of 132 floats, so the
// 16-byte reads of a warp hit distinct banks), and accumulates 4 rows x 4
// head elements of the weighted sum.
constexpr int kPfChunk = 32;
constexpr int kPfRing = 3;
constexpr int kPfRows = 32;
constexpr int kPfPitch = 132;  // floats per row of widened keys and of q
constexpr int kPfEPitch = 36;  // floats per key row of the exponentials ([key][row])
constexpr size_t kPfSlot = (size_t)kPfChunk * 128 * 2;  // f16 keys or values of a chunk
constexpr size_t kPfSmem = 128 + kPfRing * kPfSlot +
                           sizeof(float) * ((size_t)kPfChunk * kPfPitch + kPfChunk * 128 + kPfRows * kPfPitch +
                                            kPfChunk * kPfEPitch);

__global__ void __launch_bounds__(256, 2) attn_prefill_kernel(AttnArgs2 a) {
    extern __shared__ __align__(128) uint8_t pf_[];
    __shared__ float rmaxw[8][kPfRows], rmax[kPfRows], rsum[kPfRows], red[kPfRows][8], tailv[kPfRows][8];
    __shared__ int rn[kPfRows];
    constexpr int D = 128;
    uint64_t *bar = (uint64_t *)pf_;
    uint8_t *ring = pf_ + 128;
    float *kf = (float *)(ring + kPfRing * kPfSlot);  // [kPfChunk][kPfPitch]
    float *vf = kf + kPfChunk * kPfPitch;             // [kPfChunk][D]
    float *qs = vf + kPfChunk * D;                    // [kPfRows][kPfPitch]
    float *es = qs + kPfRows * kPfPitch;              // [kPfChunk][kPfEPitch]
    const int G = a.H / a.Hkv, PQ = kPfRows / G;
    const int kv = blockIdx.x, t0 = blockIdx.y * PQ, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        for (int b = 0; b < kPfRing; b++) mbar_init(&bar[b], 1);
        fence_barrier_init();
    }
    __syncthreads();
    pdl_launch_dependents();
    pdl_wait();
    // row r: query t0 + r / G, head kv*G + r % G; keys [0, n_r) (0 past the last query)
    if (tid < kPfRows) {
        const int t = t0 + tid / G;
        rn[tid] = t < a.T ? (int)(a.pos[t] + 1) : 0;
    }
    for (int i = tid; i < kPfRows * D; i += 256) {
        const int r = i / D, t = t0 + r / G, h = kv * G + r % G;
        qs[r * kPfPitch + i % D] = t < a.T ? a.qh[((long long)h * a.T + t) * D + i % D] : 0.f;
    }
    __syncthreads();
    int nmax = 0, nmin = 1 << 30;  // over the rows of real queries
    for (int r = 0; r < kPfRows; r++)
        if (rn[r] > 0) {
            nmax = max(nmax, rn[r]);
            nmin = min(nmin, rn[r]);
        }
    const int nch = (nmax + kPfChunk - 1) / kPfChunk, items = 2 * nch;
    float *srow = a.scores + (size_t)(kv * gridDim.y + blockIdx.y) * kPfRows * a.C;  // [kPfRows][C]
    const size_t slot_off = (size_t)a.slot0 * cache_slot_elems(a.Hkv, a.C, D) * 2;
    const uint8_t *kbase = (const uint8_t *)a.kc + slot_off + (size_t)kv * a.C * D * 2;
    const uint8_t *vbase = (const uint8_t *)a.vc + slot_off + (size_t)kv * a.C * D * 2;
    // item i < nch: keys of chunk i (pass 1); else values of chunk i - nch (pass 2)
    auto issue = [&](int i) {
        const int b = i % kPfRing, c = i % nch, j0 = c * kPfChunk, len = min(kPfChunk, nmax - j0);
        const uint32_t bytes = (uint32_t)(len * D * 2);
        mbar_arrive_expect_tx(&bar[b], bytes);
        bulk_g2s(ring + b * kPfSlot, (i < nch ? kbase : vbase) + (size_t)j0 * D * 2, bytes, &bar[b]);
    };
    if (tid == 0)
        for (int i = 0; i < min(items, kPfRing); i++) issue(i);
    // scoring lane: rows rg + 8i (i < 4), key jj of the chunk
    const int rg = lane & 7, jj = 4 * warp + (lane >> 3);
    auto scores = [&](int j0, float (&s)[4]) {
        float l8[4][8];
#pragma unroll
        for (int q = 0; q < 4; q++)
#pragma unroll
            for (int l = 0; l < 8; l++) l8[q][l] = 0.f;
        const float *kr = kf + jj * kPfPitch;
#pragma unroll 2
        for (int c8 = 0; c8 < D / 8; c8++) {
            const float4 k0 = *(const float4 *)(kr + 8 * c8), k1 = *(const float4 *)(kr + 8 * c8 + 4);
            const float kv8[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const float *qr = qs + (rg + 8 * q) * kPfPitch + 8 * c8;
                const float4 q0 = *(const float4 *)qr, q1 = *(const float4 *)(qr + 4);
                const float qv[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
                for (int l = 0; l < 8; l++) l8[q][l] = __fmaf_rn(qv[l], kv8[l], l8[q][l]);
            }
        }
        const int j = j0 + jj;
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int n4 = rn[rg + 8 * q] & ~3;
            const float v =
                j < n4 ? __fadd_rn(__fadd_rn(__fadd_rn(l8[q][0], l8[q][1]), __fadd_rn(l8[q][2], l8[q][3])),
                                   __fadd_rn(__fadd_rn(l8[q][4], l8[q][5]), __fadd_rn(l8[q][6], l8[q][7])))
                       : __fadd_rn(__fadd_rn(__fadd_rn(l8[q][0], l8[q][4]), __fadd_rn(l8[q][1], l8[q][5])),
                                   __fadd_rn(__fadd_rn(l8[q][2], l8[q][6]), __fadd_rn(l8[q][3], l8[q][7])));
            s[q] = __fmul_rn(v, a.scale);
        }
    };
    // widen the f16 chunk in slot b into kf (keys) or vf (values)
    auto widen = [&](int b, int len, bool values) {
        const uint32_t *k16 = (const uint32_t *)(ring + b * kPfSlot);
        float *dst = values ? vf : kf;
        const int pitch = values ? D : kPfPitch;
        for (int i = tid; i < kPfChunk * D / 2; i += 256) {
            const int kj = i / (D / 2), d2 = i % (D / 2);
            const uint32_t w = kj < len ? k16[i] : 0u;
            *(float2 *)(dst + kj * pitch + 2 * d2) = make_float2(h2f_bits(w & 0xFFFFu), h2f_bits(w >> 16));
        }
    };
    bool ok = true;
    // ---- pass 1: each row's maximum score (exact in any order)
    float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    for (int c = 0; c < nch; c++) {
        const int b = c % kPfRing, j0 = c * kPfChunk, len = min(kPfChunk, nmax - j0);
        ok &= mbar_wait_bounded(&bar[b], (c / kPfRing) & 1, a.status);
        widen(b, len, false);
        __syncthreads();  // widened; slot b free
        if (tid == 0 && c + kPfRing < items) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(c + kPfRing);
        }
        float s[4];
        scores(j0, s);
#pragma unroll
        for (int q = 0; q < 4; q++)
            if (j0 + jj < rn[rg + 8 * q]) {
                m4[q] = fmaxf(m4[q], s[q]);
                srow[(size_t)(rg + 8 * q) * a.C + j0 + jj] = s[q];  // read back by this thread in pass 2
            }
        __syncthreads();  // kf read by every warp before the next widening
    }
#pragma unroll
    for (int q = 0; q < 4; q++) {  // lanes rg, rg+8, rg+16, rg+24 hold the same rows
        float m = m4[q];
        m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 8));
        m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 16));
        if (lane < 8) rmaxw[warp][rg + 8 * q] = m;
    }
    __syncthreads();
    if (tid < kPfRows) {
        float m = rmaxw[0][tid];
        for (int w = 1; w < 8; w++) m = fmaxf(m, rmaxw[w][tid]);
        rmax[tid] = m;
    }
    __syncthreads();
    // ---- pass 2: exponentials, their sums and the weighted sum of the values
    const int sr = tid >> 3, sl = tid & 7;  // summing thread: row sr, ExpSumF32 lane sl
    const int srn = rn[sr], srn8 = srn >= 8 ? (srn & ~7) : 0;
    float lanesum = 0.f;
    int ntail = 0;
    const int ar = 4 * (lane & 7), ad = 4 * (4 * warp + (lane >> 3));  // accumulating thread: rows ar.., d ad..
    int an[4];
#pragma unroll
    for (int ri = 0; ri < 4; ri++) an[ri] = rn[ar + ri];
    float acc[4][4];
#pragma unroll
    for (int ri = 0; ri < 4; ri++)
#pragma unroll
        for (int di = 0; di < 4; di++) acc[ri][di] = 0.f;
    for (int c = 0; c < nch; c++) {
        const int i = nch + c, b = i % kPfRing, j0 = c * kPfChunk, len = min(kPfChunk, nmax - j0);
        const int j = j0 + jj;
        float s[4];
#pragma unroll
        for (int q = 0; q < 4; q++) s[q] = j < rn[rg + 8 * q] ? srow[(size_t)(rg + 8 * q) * a.C + j] : 0.f;
        ok &= mbar_wait_bounded(&bar[b], (i / kPfRing) & 1, a.status);
        widen(b, len, true);
        __syncthreads();
        if (tid == 0 && i + kPfRing < items) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(i + kPfRing);
        }
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int r = rg + 8 * q, n = rn[r], n8 = n >= 8 ? (n & ~7) : 0;
            float e = 0.f;
            if (j < n) {
                const float x = __fsub_rn(s[q], rmax[r]);
                e = j < n8 ? expf_amd64(x) : (float)exp((double)x);
            }
            es[jj * kPfEPitch + r] = e;
        }
        __syncthreads();
        // ExpSumF32's lane sums: key j to lane j % 8 below n8 (j0 is a multiple of 8), in key order
        for (int k = sl; k < len; k += 8)
            if (j0 + k < srn8) lanesum = __fadd_rn(lanesum, es[k * kPfEPitch + sr]);
        if (sl == 0)  // the tail keys [n8, n), kept in order
            for (int k = 0; k < len; k++) {
                const int jg = j0 + k;
                if (jg >= srn8 && jg < srn) tailv[sr][ntail++] = es[k * kPfEPitch + sr];
            }
        // one fused multiply-add per key and element, in key order; keys every row
        // of the block admits first, the others only for the rows that admit them
        const int kall = min(len, max(0, nmin - j0));
        for (int k = 0; k < kall; k++) {
            const float4 e4 = *(const float4 *)(es + k * kPfEPitch + ar);
            const float4 v4 = *(const float4 *)(vf + k * D + ad);
            const float ev[4] = {e4.x, e4.y, e4.z, e4.w}, vv[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
            for (int ri = 0; ri < 4; ri++)
#pragma unroll
                for (int di = 0; di < 4; di++) acc[ri][di] = __fmaf_rn(ev[ri], vv[di], acc[ri][di]);
        }
        for (int k = kall; k < len; k++) {
            const float4 e4 = *(const float4 *)(es + k * kPfEPitch + ar);
            const float4 v4 = *(const float4 *)(vf + k * D + ad);
            const float ev[4] = {e4.x, e4.y, e4.z, e4.w}, vv[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
            for (int ri = 0; ri < 4; ri++)
                if (j0 + k < an[ri])
#pragma unroll
                    for (int di = 0; di < 4; di++) acc[ri][di] = __fmaf_rn(ev[ri], vv[di], acc[ri][di]);
        }
        __syncthreads();  // es, kf, vf free
    }
    red[sr][sl] = lanesum;
    __syncthreads();
    if (sl == 0) {
        const float *r8 = red[sr];
        float sum = 0.f;
        if (srn8) sum = __fadd_rn(__fadd_rn(__fadd_rn(r8[0], r8[4]), __fadd_rn(r8[1], r8[5])),
                                  __fadd_rn(__fadd_rn(r8[2], r8[6]), __fadd_rn(r8[3], r8[7])));
        for (int k = 0; k < ntail; k++) sum = __fadd_rn(sum, tailv[sr][k]);
        rsum[sr] = sum;
    }
    __syncthreads();
    (void)ok;
#pragma unroll
    for (int ri = 0; ri < 4; ri++) {
        const int r = ar + ri, t = t0 + r / G, h = kv * G + r % G;
        if (t >= a.T) continue;
        const float sum = rsum[r];
        const float4 o = make_float4(__fdiv_rn(acc[ri][0], sum), __fdiv_rn(acc[ri][1], sum),
                                     __fdiv_rn(acc[ri][2], sum), __fdiv_rn(acc[ri][3], sum));
        *(float4 *)(a.out + (long long)t * a.H * D + (long long)h * D + ad) = o;
    }
}

// After the argmax of a greedy step: the picked id (0 when the first logit
// is NaN -- the all-ones key -- or nothing was picked) becomes the next input
// token, is appended to the output ids, the position advances, and the key
// is cleared for the next step; one thread per sequence of a batched step
// (ids [step][rows]).
__global__ void advance_kernel(unsigned long long *key, int32_t *tok, int64_t *pos, int32_t *ids, int *step,
                               P2P wait, const unsigned long long *keys, int rows) {
    pdl_wait();
    const int r = threadIdx.x;
    unsigned long long k = r < rows ? key[r] : 0ull;
    if (wait.N > 1) {  // tensor parallelism (one row): this rank's key to every rank, then the largest wins
        if (r == 0) {
            for (int q = 0; q < wait.N; q++) peer_ptr<unsigned long long>(wait, q, wait.off)[wait.k] = k;
            p2p_publish_wait(wait);
            k = 0;
            for (int q = 0; q < wait.N; q++) k = max(k, ((volatile const unsigned long long *)keys)[q]);
        }
    }
    const int s0 = *step;
    __syncthreads();
    if (r < rows) {
        const int id = (k == 0 || k == ~0ull) ? 0 : (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
        key[r] = 0;
        tok[r] = id;
        ids[(long long)s0 * rows + r] = id;
        pos[r] += 1;
    }
    if (r == 0) *step = s0 + 1;
}

}  // namespace

cudaError_t launch_rope_scatter(const RopeScatterArgs &a, cudaStream_t st, bool pdl) {
    if (a.T <= 0) return cudaSuccess;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = mk(dim3(a.T, a.H + 2 * a.Hkv), dim3((a.D + 31) / 32 * 32), 0, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, rope_scatter_kernel, a);
}

bool attn_prefill_ok(const AttnArgs2 &a) {
    return a.T >= kAttnPrefillMinRows && a.cache_f16 && a.D == 128 && a.Hkv > 0 && a.H % a.Hkv == 0 &&
           kPfRows % (a.H / a.Hkv) == 0 && !a.act.q && a.scores && !a.slot;
}

size_t attn_prefill_scores_bytes(int T, int H, int Hkv, int C) {
    if (Hkv <= 0 || H % Hkv || kPfRows % (H / Hkv)) return 0;
    const int PQ = kPfRows / (H / Hkv);
    return (size_t)Hkv * ((T + PQ - 1) / PQ) * kPfRows * C * sizeof(float);
}

cudaError_t launch_attn_prefill(const AttnArgs2 &a, cudaStream_t st, bool pdl) {
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPfSmem);
        if (e != cudaSuccess) return e;
        attr = true;
    }
    const int PQ = kPfRows / (a.H / a.Hkv);
    cudaLaunchAttribute attr1[1];
    cudaLaunchConfig_t cfg = mk(dim3(a.Hkv, (a.T + PQ - 1) / PQ), dim3(256), kPfSmem, st, pdl, attr1);
    return cudaLaunchKernelEx(&cfg, attn_prefill_kernel, a);
}

cudaError_t launch_attn_exact(const AttnArgs2 &a, cudaStream_t st, bool pdl) {
    if (a.T <= 0) return cudaSuccess;
    if (attn_prefill_ok(a)) return launch_attn_prefill(a, st, pdl);
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
                           cudaStream_t st, bool pdl, const P2P *wait, const unsigned long long *keys, int rows) {
    if (rows < 1 || rows > 1024 || (wait && wait->N > 1 && rows != 1)) return cudaErrorInvalidValue;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = mk(dim3(1), dim3((rows + 31) / 32 * 32), 0, st, pdl, attr);
    const P2P w = wait ? *wait : P2P{};
    return cudaLaunchKernelEx(&cfg, advance_kernel, key, tok, pos, ids, step, w, keys, rows);
}

}  // namespace mimgpu
