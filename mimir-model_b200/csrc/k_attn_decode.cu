// k_attn_decode.cu -- the attention of a decode step on sm_100a: RoPE of the
// token's query and key heads, the key/value cache write and attention.v2
// over the cache, fused with the 8-bit quantization of its output, in one
// kernel per layer (importer/llama.go:400-534 of gsoultan/mimir-model).
//
// Same bits as rope_scatter_kernel followed by attn_exact_kernel
// (k_model.cu): RoPE as fastRope (interp/fast.go:507-557) with the float64
// cos/sin of pos * inv_freq rounded to f32 (the session's table), the key
// and value rows rounded to the f16 cache (prim.go:76-96), and attendRow
// (interp/fast.go:728-751) with the reference's amd64 kernels: scores in the
// eight-lane orders of scoresF16AVX2, ExpSumF32 (Cephes expf on the first
// n&~7 keys and its lane-sum order, float64 exp on the rest), the
// key-ordered fused weighted sum of wsumF16AVX2, o = acc/sum.
//
// A block takes two query heads of one token (one kv head: the group size
// must be even), or four in a batched grid that still has a block for every
// SM and a group size divisible by four, and 256 threads.  Decode attention
// is latency-bound (a few blocks per token), so the layout minimises serial
// steps:
//  * The keys and values of earlier tokens stream through a ring of chunk
//    buffers, requested BEFORE the grid dependency wait: they were written by
//    earlier steps, all complete once this step's first kernel (the
//    embedding) has passed its own wait, and nothing in this step writes them.
//    The token's own key and value rows are made here (RoPE, f16) and read
//    from shared memory, never from the cache.
//  * The chunk size is chosen at launch.  A grid of at most one block per
//    SM (one token) takes 256-key chunks: few serial steps.  A larger grid
//    (batched decode), or a context whose scores leave no room for two 64 KB
//    buffers, takes 128-key chunks, so that three blocks share an SM and one
//    block's serial phases (softmax, the key-ordered weighted sum) overlap
//    the others' copies.
//  * A key chunk is two 3-D tensor copies (TMA) of [CH keys][64 elements] in
//    the 128-byte swizzle (one map per chunk size), so the 16-byte loads of
//    eight consecutive keys at one column hit eight distinct bank groups; a
//    value chunk is one bulk copy of dense rows.  A thread scores one key
//    with the whole row unrolled: for both heads in a 256-key chunk, for one
//    head (threads 0-127 the first) in a 128-key chunk of two heads, for two
//    heads (threads 0-127 heads 0-1, 128-255 heads 2-3) in one of four.
//  * The weighted sum: 64 threads per head, two output elements each, with
//    the exponentials and value pairs of eight keys loaded ahead of the
//    fused multiply-adds.
// The scores of the block's heads over the whole context live in shared
// memory (context <= attn_decode_max_context()).
#include "common.cuh"
#include "model_kernels.h"
#include "amd64_math.cuh"
#include "quant.cuh"
#include "p2p.cuh"

namespace mimgpu {

namespace {

constexpr int kD = 128;               // head elements
constexpr int kRing = 2;              // chunk buffers (one mbarrier each, below kOffQ)
// CH keys per chunk: a buffer holds a key chunk (two swizzled 64-element
// halves of CH rows) or a value chunk (CH dense rows)
template <int CH> constexpr int slot_bytes() { return CH * kD * 2; }
// Shared layout of a block of HPB query heads: mbarriers, the queries (then
// the outputs) [HPB][kD] f32, the token's key and value rows f16, the
// softmax's lane sums [HPB][8], maxima [HPB] and sums [HPB], the
// quantization scratch, then the chunk ring (1024-byte aligned for the
// swizzle) and the scores [HPB][C].
constexpr int kOffQ = 64;
template <int HPB> struct Lay {
    static constexpr int kOffNew = kOffQ + HPB * kD * 4, kOffRed = kOffNew + 2 * kD * 2;
    static constexpr int kOffQs = HPB == 2 ? 1792 : 2816, kOffRing = HPB == 2 ? 2048 : 3072;
    static_assert(kOffRed + 10 * HPB * 4 <= kOffQs && kOffQs + (int)sizeof(QuantScratch) <= kOffRing,
                  "shared layout");
    static_assert(kOffRing % 1024 == 0, "swizzled ring alignment");
};
static_assert(kRing * 8 <= kOffQ, "mbarriers below the query");
constexpr int kSmemCap = 226 * 1024;  // + the static quantization scratch
constexpr unsigned FULLM = 0xffffffffu;

__host__ __device__ inline int sc_stride(int C) { return (C + 3) & ~3; }
__host__ __device__ inline size_t dec_smem(int C, int ch, int hpb) {
    return (size_t)(hpb == 2 ? Lay<2>::kOffRing : Lay<4>::kOffRing) + (size_t)kRing * ch * kD * 2 +
           (size_t)hpb * sc_stride(C) * 4;
}

// Element e of one RoPE'd head (rope.v1, fast.go:507-557): pairs (i, i + r/2)
// or (2i, 2i + 1), cs[i] = (f32(cos), f32(sin)) of pos * inv_freq[i].
__device__ __forceinline__ float rope_elem(const float *src, int e, int rotary, int interleaved, const float2 *cs,
                                           uint64_t keep) {
    if (e >= rotary) return src[e];
    const int h2 = rotary / 2;
    int i, first;
    if (interleaved) {
        i = e >> 1;
        first = !(e & 1);
    } else {
        i = e < h2 ? e : e - h2;
        first = e < h2;
    }
    const int i1 = interleaved ? 2 * i : i, i2 = interleaved ? 2 * i + 1 : i + h2;
    const float2 c = ldg_keep2(cs + i, keep);  // the table stays in L2 across steps
    const float x1 = src[i1], x2 = src[i2];
    return first ? __fsub_rn(__fmul_rn(x1, c.x), __fmul_rn(x2, c.y)) : __fadd_rn(__fmul_rn(x2, c.x), __fmul_rn(x1, c.y));
}

__device__ __forceinline__ void fma8(float (&l8)[8], const float4 q0, const float4 q1, const uint4 w) {
    l8[0] = __fmaf_rn(q0.x, h2f_bits(w.x & 0xFFFFu), l8[0]);
    l8[1] = __fmaf_rn(q0.y, h2f_bits(w.x >> 16), l8[1]);
    l8[2] = __fmaf_rn(q0.z, h2f_bits(w.y & 0xFFFFu), l8[2]);
    l8[3] = __fmaf_rn(q0.w, h2f_bits(w.y >> 16), l8[3]);
    l8[4] = __fmaf_rn(q1.x, h2f_bits(w.z & 0xFFFFu), l8[4]);
    l8[5] = __fmaf_rn(q1.y, h2f_bits(w.z >> 16), l8[5]);
    l8[6] = __fmaf_rn(q1.z, h2f_bits(w.w & 0xFFFFu), l8[6]);
    l8[7] = __fmaf_rn(q1.w, h2f_bits(w.w >> 16), l8[7]);
}

// 3-D tensor copy [x elements][y keys][z head] of the key cache into shared
// memory (1024-byte aligned for the 128-byte swizzle); x is 0 or 64 (a
// 16-byte multiple of bytes).
__device__ __forceinline__ void tma_3d(const CUtensorMap *map, uint8_t *dst, int x, int y, int z, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(dst)),
        "l"((const void *)map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

// Three 128-key blocks of two heads share an SM when a thread holds at most
// 80 registers (that instance uses fewer; -Xptxas -v shows it); blocks of
// four heads take twice the scores and fit two to an SM.
template <int CH, int HPB>
__global__ void __launch_bounds__(256) attn_decode_kernel(const __grid_constant__ AttnDecodeArgs p) {
    static_assert(CH == 128 || CH == 256, "chunk of one key per thread and head, or per thread");
    static_assert(HPB == 2 || (HPB == 4 && CH == 128), "two heads a block, or four with 128-key chunks");
    constexpr int kSlot = slot_bytes<CH>(), kHalf = CH * 128, kCh = CH;
    constexpr int kOffNew = Lay<HPB>::kOffNew, kOffRed = Lay<HPB>::kOffRed, kOffQs = Lay<HPB>::kOffQs,
                  kOffRing = Lay<HPB>::kOffRing;
    // No static shared memory: the dynamic block starts at the CTA's shared
    // base, so the swizzled key chunks at kOffRing are 1024-byte aligned.
    extern __shared__ __align__(1024) uint8_t sm[];
    QuantScratch &qs = *(QuantScratch *)(sm + kOffQs);
    const AttnArgs2 &a = p.at;
    uint64_t *bar = (uint64_t *)sm;
    float *q = (float *)(sm + kOffQ);                  // [HPB][kD]; the outputs at the end
    uint16_t *knew = (uint16_t *)(sm + kOffNew), *vnew = knew + kD;
    float *red = (float *)(sm + kOffRed);              // [HPB][8] lane sums, then max[HPB], sum[HPB]
    float *hmax = red + 8 * HPB, *hsum = hmax + HPB;
    uint8_t *ring = sm + kOffRing;
    const int ldsc = sc_stride(a.C);
    constexpr int R = kRing;
    float *sc = (float *)(sm + kOffRing + R * kSlot);  // [HPB][ldsc]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int t = blockIdx.y, h0 = HPB * blockIdx.x, G = a.H / a.Hkv, kvh = h0 / G;
    // the 128-byte swizzle needs a 1024-byte aligned destination: a block
    // placed otherwise reports DEV_BADARG and copies nothing
    if (smem_u32(ring) & 1023u) {
        if (tid == 0 && a.status) atomicOr(a.status, (unsigned)DEV_BADARG);
        pdl_launch_dependents();
        return;
    }
    if (tid == 0) {
        for (int b = 0; b < R; b++) mbar_init(&bar[b], 1);
        fence_barrier_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    // ---- before the wait: the earlier tokens' keys and values
    const long long pos = a.pos[t];
    const int n = (int)pos + 1;
    const int nch = (n + kCh - 1) / kCh, items = 2 * nch;  // key chunks, then value chunks
    const int seq = a.slot ? a.slot[t] : a.slot0;
    const long long slot_elems = (long long)seq * cache_slot_elems(a.Hkv, a.C, kD);
    const long long head_off = slot_elems + (long long)kvh * a.C * kD;
    const uint16_t *vbase = (const uint16_t *)a.vc + head_off;
    // item i into buffer i % R (lane 0 of warp 0): key chunk i (two
    // swizzled halves; rows past the context come as zeros) or value chunk
    // i - nch (rows [j0, n - 1): the token's own row is made here)
    auto issue = [&](int i) {
        const int b = i % R;
        uint8_t *dst = ring + (size_t)b * kSlot;
        if (i < nch) {
            mbar_arrive_expect_tx(&bar[b], (uint32_t)kSlot);
            tma_3d(&p.kmap[CH == 256 ? 0 : 1], dst, 0, i * kCh, seq * a.Hkv + kvh, &bar[b]);
            tma_3d(&p.kmap[CH == 256 ? 0 : 1], dst + kHalf, 64, i * kCh, seq * a.Hkv + kvh, &bar[b]);
            return;
        }
        const int j0 = (i - nch) * kCh, len = min(kCh, n - 1 - j0);
        if (len <= 0) {  // the chunk holds only the token's own row
            mbar_arrive(&bar[b]);
            return;
        }
        mbar_arrive_expect_tx(&bar[b], (uint32_t)len * (kD * 2));
        bulk_g2s(dst, vbase + (long long)j0 * kD, (uint32_t)len * (kD * 2), &bar[b]);
    };
    if (tid == 0)
        for (int i = 0; i < min(items, R); i++) issue(i);

    // ---- after the wait: the token's q, k, v (the QKV product)
    pdl_wait();
    const float *row = p.qkv + (long long)t * p.ldq;
    const float2 *cs = p.rope_cs + pos * (p.rotary / 2);
    const uint64_t keep = l2_policy_evict_last();
    if constexpr (HPB == 2) {
        const int hh = tid >> 7, e = tid & (kD - 1);
        q[hh * kD + e] = rope_elem(row + (long long)(h0 + hh) * kD, e, p.rotary, p.interleaved, cs, keep);
    } else {
#pragma unroll
        for (int u = 0; u < HPB / 2; u++) {
            const int hh = 2 * u + (tid >> 7), e = tid & (kD - 1);
            q[hh * kD + e] = rope_elem(row + (long long)(h0 + hh) * kD, e, p.rotary, p.interleaved, cs, keep);
        }
    }
    const bool writer = h0 % G == 0;  // one block of each kv group writes the cache rows
    const long long at = head_off + pos * kD;
    if (tid < kD) {
        const uint16_t h = f32_to_f16(rope_elem(row + (long long)(a.H + kvh) * kD, tid, p.rotary, p.interleaved, cs, keep));
        knew[tid] = h;
        if (writer) ((uint16_t *)a.kc)[at + tid] = h;
    } else {
        const int e = tid - kD;
        const uint16_t h = f32_to_f16(row[(long long)(a.H + a.Hkv + kvh) * kD + e]);
        vnew[e] = h;
        if (writer) ((uint16_t *)a.vc)[at + e] = h;
    }
    __syncthreads();

    // ---- scores: a 256-key chunk takes key tid for both heads; a 128-key
    // chunk of two heads key tid % 128 for head tid / 128, of four heads key
    // tid % 128 for heads 2 (tid / 128) and 2 (tid / 128) + 1
    bool ok = true;
    const int n4 = n & ~3;
    if constexpr (CH == 256 || HPB == 4) {
        const uint32_t knew_s = smem_u32(knew), ring_s = smem_u32(ring);
        const int hb = CH == 256 ? 0 : 2 * (tid >> 7);  // the thread's first head
        const float *q0 = q + hb * kD, *q1 = q0 + kD;
        float *sc0 = sc + hb * ldsc;
        for (int c = 0; c < nch; c++) {
            const int b = c % R, jj = CH == 256 ? tid : tid & (kCh - 1), j = c * kCh + jj;
            ok &= mbar_wait_bounded(&bar[b], (c / R) & 1, a.status);
            if (j < n) {
                // 16-byte unit c8 of key jj: half c8/8, row jj, swizzled unit (c8 % 8) ^ (jj % 8)
                const bool own = j == n - 1;
                const uint32_t kb = ring_s + (uint32_t)(b * kSlot + jj * 128), sw = (uint32_t)(jj & 7);
                float la[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, lb[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int c8 = 0; c8 < kD / 8; c8++) {
                    const uint32_t addr = own ? knew_s + 16 * c8
                                              : kb + (uint32_t)((c8 >> 3) * kHalf) + ((((uint32_t)c8 & 7) ^ sw) << 4);
                    uint4 w;
                    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(w.x), "=r"(w.y), "=r"(w.z), "=r"(w.w) : "r"(addr));
                    fma8(la, *(const float4 *)(q0 + 8 * c8), *(const float4 *)(q0 + 8 * c8 + 4), w);
                    fma8(lb, *(const float4 *)(q1 + 8 * c8), *(const float4 *)(q1 + 8 * c8 + 4), w);
                }
                const float va = j < n4 ? __fadd_rn(__fadd_rn(__fadd_rn(la[0], la[1]), __fadd_rn(la[2], la[3])),
                                                    __fadd_rn(__fadd_rn(la[4], la[5]), __fadd_rn(la[6], la[7])))
                                        : __fadd_rn(__fadd_rn(__fadd_rn(la[0], la[4]), __fadd_rn(la[1], la[5])),
                                                    __fadd_rn(__fadd_rn(la[2], la[6]), __fadd_rn(la[3], la[7])));
                const float vb = j < n4 ? __fadd_rn(__fadd_rn(__fadd_rn(lb[0], lb[1]), __fadd_rn(lb[2], lb[3])),
                                                    __fadd_rn(__fadd_rn(lb[4], lb[5]), __fadd_rn(lb[6], lb[7])))
                                        : __fadd_rn(__fadd_rn(__fadd_rn(lb[0], lb[4]), __fadd_rn(lb[1], lb[5])),
                                                    __fadd_rn(__fadd_rn(lb[2], lb[6]), __fadd_rn(lb[3], lb[7])));
                sc0[j] = __fmul_rn(va, a.scale);
                sc0[ldsc + j] = __fmul_rn(vb, a.scale);
            }
            __syncthreads();  // every thread is done with buffer b
            if (tid == 0 && c + R < items) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                issue(c + R);
            }
        }
    } else {
        const uint32_t knew_s = smem_u32(knew), ring_s = smem_u32(ring);
        const int hh = tid >> 7, jj = tid & (kCh - 1);
        const float *qh = q + hh * kD;
        float *sch = sc + hh * ldsc;
        const uint32_t sw = (uint32_t)(jj & 7);
        for (int c = 0; c < nch; c++) {
            const int b = c % R, j = c * kCh + jj;
            ok &= mbar_wait_bounded(&bar[b], (c / R) & 1, a.status);
            if (j < n) {
                const bool own = j == n - 1;
                const uint32_t kb = ring_s + (uint32_t)(b * kSlot + jj * 128);
                float la[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int c8 = 0; c8 < kD / 8; c8++) {
                    const uint32_t addr = own ? knew_s + 16 * c8
                                              : kb + (uint32_t)((c8 >> 3) * kHalf) + ((((uint32_t)c8 & 7) ^ sw) << 4);
                    uint4 w;
                    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(w.x), "=r"(w.y), "=r"(w.z), "=r"(w.w) : "r"(addr));
                    fma8(la, *(const float4 *)(qh + 8 * c8), *(const float4 *)(qh + 8 * c8 + 4), w);
                }
                const float va = j < n4 ? __fadd_rn(__fadd_rn(__fadd_rn(la[0], la[1]), __fadd_rn(la[2], la[3])),
                                                    __fadd_rn(__fadd_rn(la[4], la[5]), __fadd_rn(la[6], la[7])))
                                        : __fadd_rn(__fadd_rn(__fadd_rn(la[0], la[4]), __fadd_rn(la[1], la[5])),
                                                    __fadd_rn(__fadd_rn(la[2], la[6]), __fadd_rn(la[3], la[7])));
                sch[j] = __fmul_rn(va, a.scale);
            }
            __syncthreads();  // every thread is done with buffer b
            if (tid == 0 && c + R < items) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                issue(c + R);
            }
        }
    }
    // ---- softmax: max per head (exact in any order)
    if (warp < HPB) {
        float m = -INFINITY;
        for (int j = lane; j < n; j += 32) m = fmaxf(m, sc[warp * ldsc + j]);
        m = warp_max(m);
        if (lane == 0) hmax[warp] = m;
    }
    __syncthreads();
    // exponentials: Cephes on the first n&~7 keys (none when n < 8), float64 on the rest
    const int n8 = n >= 8 ? (n & ~7) : 0;
#pragma unroll
    for (int hh = 0; hh < HPB; hh++)
        for (int j = tid; j < n; j += 256) {
            const float x = __fsub_rn(sc[hh * ldsc + j], hmax[hh]);
            sc[hh * ldsc + j] = j < n8 ? expf_amd64(x) : (float)exp((double)x);
        }
    __syncthreads();
    // ExpSumF32's sum: eight lane sums in key order, combined, then the tail in order
    if (tid < 8 * HPB) {
        const int hh = tid >> 3, ll = tid & 7;
        const float *e = sc + hh * ldsc;
        float sl = 0.f;
#pragma unroll 8
        for (int j = ll; j < n8; j += 8) sl = __fadd_rn(sl, e[j]);
        red[hh * 8 + ll] = sl;
    }
    __syncthreads();
    if (tid < HPB) {
        const float *r = red + tid * 8;
        float sum = 0.f;
        if (n8) sum = __fadd_rn(__fadd_rn(__fadd_rn(r[0], r[4]), __fadd_rn(r[1], r[5])),
                                __fadd_rn(__fadd_rn(r[2], r[6]), __fadd_rn(r[3], r[7])));
        for (int j = n8; j < n; j++) sum = __fadd_rn(sum, sc[tid * ldsc + j]);
        hsum[tid] = sum;
    }
    // ---- weighted sum of the values, one fused multiply-add per key in key
    // order: thread tid < 64 HPB takes elements d0, d0 + 1 of head tid / 64
    const int hw = tid >> 6, d0 = (tid & 63) * 2;
    const float *e = sc + hw * ldsc;
    float acc0 = 0.f, acc1 = 0.f;
    for (int c = 0; c < nch; c++) {
        const int i = nch + c, b = i % R, j0 = c * kCh;
        ok &= mbar_wait_bounded(&bar[b], (i / R) & 1, a.status);
        if (tid < 64 * HPB) {
            const uint8_t *vb = ring + (size_t)b * kSlot + d0 * 2;
            const int lc = min(kCh, n - 1 - j0);  // rows from the ring (the token's own row after them)
            int jj = 0;
            for (; jj + 8 <= lc; jj += 8) {
                const float4 ea = *(const float4 *)(e + j0 + jj), eb = *(const float4 *)(e + j0 + jj + 4);
                uint32_t v[8];
#pragma unroll
                for (int u = 0; u < 8; u++) v[u] = *(const uint32_t *)(vb + (size_t)(jj + u) * (kD * 2));
                const float ev[8] = {ea.x, ea.y, ea.z, ea.w, eb.x, eb.y, eb.z, eb.w};
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    acc0 = __fmaf_rn(ev[u], h2f_bits(v[u] & 0xFFFFu), acc0);
                    acc1 = __fmaf_rn(ev[u], h2f_bits(v[u] >> 16), acc1);
                }
            }
            for (; jj < lc; jj++) {
                const uint32_t v = *(const uint32_t *)(vb + (size_t)jj * (kD * 2));
                acc0 = __fmaf_rn(e[j0 + jj], h2f_bits(v & 0xFFFFu), acc0);
                acc1 = __fmaf_rn(e[j0 + jj], h2f_bits(v >> 16), acc1);
            }
            if (j0 + kCh >= n) {  // the last chunk: the token's own row
                acc0 = __fmaf_rn(e[n - 1], h2f_bits(vnew[d0]), acc0);
                acc1 = __fmaf_rn(e[n - 1], h2f_bits(vnew[d0 + 1]), acc1);
            }
        }
        __syncthreads();
        if (tid == 0 && i + R < items) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(i + R);
        }
    }
    (void)ok;  // a wait that ran out has set DEV_TIMEOUT in *status: the host reports it
    // ---- outputs: o = acc / sum, in element order through shared memory
    if (tid < 64 * HPB) {
        q[hw * kD + d0] = __fdiv_rn(acc0, hsum[hw]);
        q[hw * kD + d0 + 1] = __fdiv_rn(acc1, hsum[hw]);
    }
    __syncthreads();
    const int E = a.H * kD;
    if constexpr (HPB == 2) {
        const float o = q[tid];
        a.out[(long long)t * E + (long long)h0 * kD + tid] = o;
        // tensor parallelism: this rank's heads into every rank's full vector
        for (int r = 0; r < (a.put.N > 1 ? a.put.N : 0); r++)
            peer_ptr<float>(a.put, r, a.put.off)[a.put.col0 + (long long)h0 * kD + tid] = o;
        if (a.put.N > 1) {
            // visible system-wide before the kernel ends (the next kernel publishes the exchange)
            __syncthreads();
            if (tid == 0) __threadfence_system();
        }
        if (a.act.q) quant_block_256(o, t, E, blockIdx.x, a.act, qs);
    } else {
        // HPB / 2 quantization blocks of 256 outputs each
#pragma unroll
        for (int u = 0; u < HPB / 2; u++) {
            const float o = q[256 * u + tid];
            a.out[(long long)t * E + (long long)h0 * kD + 256 * u + tid] = o;
            for (int r = 0; r < (a.put.N > 1 ? a.put.N : 0); r++)
                peer_ptr<float>(a.put, r, a.put.off)[a.put.col0 + (long long)h0 * kD + 256 * u + tid] = o;
        }
        if (a.put.N > 1) {
            __syncthreads();
            if (tid == 0) __threadfence_system();
        }
        if (a.act.q) {
#pragma unroll
            for (int u = 0; u < HPB / 2; u++) {
                if (u) __syncthreads();  // the scratch of the previous block is read
                quant_block_256(q[256 * u + tid], t, E, (HPB / 2) * blockIdx.x + u, a.act, qs);
            }
        }
    }
}

}  // namespace

void *tmap_encode_fn();  // cuTensorMapEncodeTiled from the driver (k_gemv_a8.cu)
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

bool attn_decode_kmap(const void *kc, int slots, int Hkv, int C, CUtensorMap out[2]) {
    const EncodeTiledFn fn = (EncodeTiledFn)tmap_encode_fn();
    if (!fn || !kc || ((uintptr_t)kc & 15) || slots <= 0 || Hkv <= 0 || C <= 0) return false;
    const cuuint64_t dims[3] = {(cuuint64_t)kD, (cuuint64_t)C, (cuuint64_t)slots * Hkv};
    const cuuint64_t strides[2] = {(cuuint64_t)kD * 2, (cuuint64_t)C * kD * 2};
    const cuuint32_t estr[3] = {1, 1, 1};
    for (int m = 0; m < 2; m++) {  // box rows: 256, then 128
        const cuuint32_t box[3] = {64, (cuuint32_t)(256 >> m), 1};
        if (fn(&out[m], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(kc), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    return true;
}

int attn_decode_max_context() {
    return (int)((kSmemCap - Lay<2>::kOffRing - (size_t)kRing * slot_bytes<128>()) / 8) & ~3;
}

// The shape of a launch: 256-key chunks and two heads a block for a grid of
// at most one block per SM whose scores leave room for two 256-key buffers;
// else 128-key chunks, so that several blocks share an SM, with four heads
// a block (each kv head's rows read into shared memory once per four query
// heads) when the group size allows, the scores fit and the grid still has
// a block for every SM.
static void decode_shape(const AttnArgs2 &a, int *ch, int *hpb) {
    const int G = a.H / a.Hkv;
    if ((a.H / 2) * a.T <= num_sms() && dec_smem(a.C, 256, 2) <= kSmemCap) {
        *ch = 256;
        *hpb = 2;
        return;
    }
    *ch = 128;
    *hpb = G % 4 == 0 && dec_smem(a.C, 128, 4) <= kSmemCap && (a.H / 4) * a.T >= num_sms() ? 4 : 2;
}

bool attn_decode_ok(const AttnArgs2 &a) {
    return a.cache_f16 && a.D == kD && a.Hkv > 0 && a.H % a.Hkv == 0 && (a.H / a.Hkv) % 2 == 0 && a.T >= 1 &&
           (a.T == 1 || a.slot != nullptr) && a.C >= 1 && a.C <= attn_decode_max_context();
}

cudaError_t launch_attn_decode(const AttnDecodeArgs &p, cudaStream_t st, bool pdl) {
    const AttnArgs2 &a = p.at;
    if (!attn_decode_ok(a) || !p.qkv || !p.rope_cs || p.rotary <= 0 || p.rotary > kD || p.rotary % 2)
        return cudaErrorInvalidValue;
    int ch = 0, hpb = 0;
    decode_shape(a, &ch, &hpb);
    const size_t smem = dec_smem(a.C, ch, hpb);
    void (*kern)(AttnDecodeArgs) = ch == 256 ? attn_decode_kernel<256, 2>
                                   : hpb == 4 ? attn_decode_kernel<128, 4> : attn_decode_kernel<128, 2>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.H / hpb, a.T);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

}  // namespace mimgpu
