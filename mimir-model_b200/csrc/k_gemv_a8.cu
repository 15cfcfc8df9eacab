// k_gemv_a8.cu -- the product of dequant_matmul_a8.v2 (block 256) on sm_100a.
//
// Bit-exact with dotQ8KRef (internal/kernels/q8k_test.go:35-117 of
// gsoultan/mimir-model): per 256-element block the exact int32 sums
// S = sum_s sc_s * sum(q*y) and (Q4_K) M = sum_s m_s * xs_s, then in block
// order tot = fma(float(S), d*dx, tot), off = fma(float(M), dmin*dx, off);
// the result is tot - off, plus the bias, plus the residual.  Rows the
// reference refuses (linearA8, interp/fast.go:282-379) take the f32 product.
//
// Work decomposition.  A consumer warp owns 8 weight rows at a time; 4
// lanes share a row and each takes a quarter of the current block (Q4_K:
// one 32-byte run of nibbles = 64 weights; Q6_K: 16 positions of one half).
// The quarter sums are combined with two xor-shuffles inside the 4-lane
// group, so every lane of the group holds the block's exact S and M and
// the block-ordered fma chain stays in registers -- no cross-lane chain.
// A CTA has 4 consumer warps and one producer thread.  The producer streams
// the rows' slices of 4 blocks (576 B of Q4_K, 840 B of Q6_K per row) into a
// 3-stage shared-memory ring with cp.async.bulk; each slice is copied from
// the 16-byte boundary below it, so rows of any length (Q6_K blocks are
// 210 bytes) keep their byte-exact layout.  The producer does not wait for
// the previous kernel (weights are read-only), so under programmatic
// dependent launch the weights stream in while that kernel finishes.  The
// activations (int8 quants, scales, sums) are copied into shared memory once
// per CTA, after the wait.
#include <cuda.h>  // CUtensorMap (types only; the encoder is fetched from the driver at run time)

#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "kernels.h"
#include "a8_refused.cuh"
#include "p2p.cuh"

namespace mimgpu {

namespace {

constexpr int kWarps = 4;                    // consumer warps per CTA
constexpr int kRowsW = 16;                   // rows per consumer warp (2 lanes per row)
constexpr int kRowsCta = kWarps * kRowsW;    // rows of one stage
constexpr int kThreads = (kWarps + 1) * 32;
constexpr int kStages = 3;
constexpr int kKC = 2;                       // blocks of 256 per row slice
constexpr int kMaxNR = 8;                    // activation rows per launch
constexpr int kActBudget = 40 * 1024;        // shared-memory bytes for activations
constexpr int kBoxMax = 432;                 // bytes per row of a 2-D TMA box (Q6_K)
constexpr unsigned FULL = 0xffffffffu;

// Bytes per row of the 2-D TMA box of a slice: Q4_K slices (288 bytes) start
// on 16-byte boundaries; a Q6_K slice (420 bytes) is boxed as 432 bytes from
// the boundary below it.  Rows land this many bytes apart in shared memory
// (432 = 108 words puts consecutive rows 12 banks apart).
__host__ __device__ constexpr int box_bytes(int dt) { return dt == Q4_K ? kKC * 144 : kBoxMax; }

struct __align__(64) A8Params {
    CUtensorMap tmap[kMaxSegs];  // 2-D maps [rows, row bytes / 8] of u64, box [box/8, 16]
    int tma2d;                   // 1: every segment has a map; 0: per-row 1-D copies
    GemvSeg seg[kMaxSegs];
    int seg_g0[kMaxSegs + 1];  // first 8-row group of each segment; [nseg] = total
    int nseg;
    const float *x;            // f32 activations (refused rows)
    ActQ8 act;
    int rows;                  // activation rows of this launch (<= NR)
    long long K;
    int nb;                    // K / 256
    int chunks;                // ceil(nb / kKC)
    int split;                 // warps sharing a row group, each a range of K
    int cpp;                   // chunks per part: ceil(chunks / split)
    int rec_bytes;             // shared bytes per part for its per-block values
    int slot;                  // 1-D mode: bytes per row slot of a stage
    int stage_bytes;           // bytes of one stage
    int act_bytes;             // shared-memory bytes of the activations
    int act_bulk;              // 1: every activation array is 16-byte aligned: one bulk copy each
    P2P put;                   // tensor parallelism: outputs also into every rank's copy, then publish
    unsigned *status;
};

// ---- shared-memory access by 32-bit shared address
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ void sts128(uint32_t a, float x, float y, float z, float w) {
    asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(a), "f"(x), "f"(y), "f"(z), "f"(w) : "memory");
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
// Dynamic shared memory header: mbarriers (bytes 0..127) and the segment
// table (from byte 128); the activations follow.
constexpr int kHeader = 512;

// The launch's matrices, copied into shared memory at CTA start so that the
// hot loops index them without dynamic accesses to the parameter space.
struct SegTable {
    GemvSeg seg[kMaxSegs];
    int g0[kMaxSegs + 1];
    int nseg;
};
static_assert(128 + sizeof(SegTable) <= kHeader, "segment table exceeds the shared-memory header");
__device__ __forceinline__ int find_seg(const SegTable &t, int g) {
    int s = 0;
    while (s + 1 < t.nseg && g >= t.g0[s + 1]) s++;
    return s;
}

// The row group of group slot gi of CTA b in round t (a CTA has kWarps /
// split slots): groups are dealt to CTAs first, so a small matrix still
// spreads over every SM.
__device__ __forceinline__ int group_of(int b, int gi, int slots, int t) { return b + gridDim.x * (gi + slots * t); }

struct ActSmem {
    uint32_t q, dx, xs, ys;  // shared addresses of each array (row-major by activation row)
};

__device__ __forceinline__ float f16f(uint32_t h) {  // f16 -> f32 by the hardware conversion (exact)
    float f;
    asm("{ .reg .b16 t; mov.b16 t, %1; cvt.f32.f16 %0, t; }" : "=f"(f) : "h"((unsigned short)h));
    return f;
}
__device__ __forceinline__ int sbyte(uint32_t w, int i) { return (int)(int8_t)((w >> (8 * i)) & 0xFF); }
__device__ __forceinline__ int ubyte(uint32_t w, int i) { return (int)((w >> (8 * i)) & 0xFF); }

// One slice (kbn blocks from global block kb0) of the lane's Q4_K row.  Lane
// half h takes qs bytes [64h, 64h+64): sub-blocks 4h..4h+3, elements
// [128h, 128h+128).  `base` is the shared address of the slice's first block
// (16-byte aligned: Q4_K blocks are 144 bytes).
template <int NR>
__device__ __forceinline__ bool q4k_slice(uint32_t base, int kbn, int kb0, const A8Params &p, const ActSmem &as,
                                          float (&tot)[NR], float (&off)[NR], uint32_t rec) {
    const int h = threadIdx.x & 1;
    bool bad = false;
#pragma unroll
    for (int bl = 0; bl < kKC; bl++) {
        if (bl >= kbn) break;
        const uint32_t blk = base + bl * 144;
        const uint4 hdr = lds128(blk);
        uint4 q[4];
#pragma unroll
        for (int i = 0; i < 4; i++) q[i] = lds128(blk + 16 + 64 * h + 16 * i);
        const uint32_t dh = hdr.x & 0xFFFFu, mh = hdr.x >> 16;
        bad |= !f16_finite(dh) || !f16_finite(mh);
        const float d = f16f(dh), dmin = f16f(mh);
        // the 4 scales and mins of sub-blocks 4h..4h+3 as packed bytes
        // (getScaleMinK4, quant.go:246-254)
        const uint32_t scw = h ? ((hdr.w & 0x0F0F0F0Fu) | (((hdr.y >> 6) & 0x03030303u) << 4)) : (hdr.y & 0x3F3F3F3Fu);
        const uint32_t mw = h ? (((hdr.w >> 4) & 0x0F0F0F0Fu) | (((hdr.z >> 6) & 0x03030303u) << 4)) : (hdr.z & 0x3F3F3F3Fu);
        const uint32_t qw[16] = {q[0].x, q[0].y, q[0].z, q[0].w, q[1].x, q[1].y, q[1].z, q[1].w,
                                 q[2].x, q[2].y, q[2].z, q[2].w, q[3].x, q[3].y, q[3].z, q[3].w};
        const int kb = kb0 + bl;
#pragma unroll
        for (int a = 0; a < NR; a++) {
            if (a >= p.rows) break;
            const uint32_t ya = as.q + (uint32_t)(a * p.K + kb * 256 + 128 * h);
            uint32_t y[32];
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const uint4 v = lds128(ya + 16 * i);
                y[4 * i] = v.x; y[4 * i + 1] = v.y; y[4 * i + 2] = v.z; y[4 * i + 3] = v.w;
            }
            int s0 = 0, s1 = 0, s2 = 0, s3 = 0;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                s0 = __dp4a((int)(qw[i] & 0x0F0F0F0Fu), (int)y[i], s0);
                s1 = __dp4a((int)((qw[i] >> 4) & 0x0F0F0F0Fu), (int)y[8 + i], s1);
                s2 = __dp4a((int)(qw[8 + i] & 0x0F0F0F0Fu), (int)y[16 + i], s2);
                s3 = __dp4a((int)((qw[8 + i] >> 4) & 0x0F0F0F0Fu), (int)y[24 + i], s3);
            }
            int S = ubyte(scw, 0) * s0 + ubyte(scw, 1) * s1 + ubyte(scw, 2) * s2 + ubyte(scw, 3) * s3;
            const uint2 xs = lds64(as.xs + (uint32_t)((a * p.K / 32 + kb * 8 + 4 * h) * 2));
            int M = ubyte(mw, 0) * (int)(int16_t)(xs.x & 0xFFFF) + ubyte(mw, 1) * (int)(int16_t)(xs.x >> 16) +
                    ubyte(mw, 2) * (int)(int16_t)(xs.y & 0xFFFF) + ubyte(mw, 3) * (int)(int16_t)(xs.y >> 16);
            S += __shfl_xor_sync(FULL, S, 1);
            M += __shfl_xor_sync(FULL, M, 1);
            const float dx = __uint_as_float(lds32(as.dx + (uint32_t)((a * p.nb + kb) * 4)));
            const float fs = __int2float_rn(S), pd = __fmul_rn(d, dx);
            const float fm = __int2float_rn(M), pm = __fmul_rn(dmin, dx);
            if (rec) {
                if (h == 0) sts128(rec + (uint32_t)(((bl * NR + a) * kRowsW) * 16), fs, pd, fm, pm);
            } else {
                tot[a] = __fmaf_rn(fs, pd, tot[a]);
                off[a] = __fmaf_rn(fm, pm, off[a]);
            }
        }
    }
    return bad;
}

// The bytes a Q6_K lane needs from one block, read with aligned 16-byte
// loads: WO is the block start's word offset within its 16-byte line
// (warp-uniform for the usual row lengths), sh the remaining 0/16-bit shift.
template <int WO>
__device__ __forceinline__ void q6k_load(uint32_t blk, int h, uint32_t (&ql)[16], uint32_t (&qh)[8], uint32_t &sc01,
                                         uint32_t &sc23, uint32_t &dh) {
    const uint32_t sh = (blk & 3u) * 8;
    const uint32_t b16 = blk & ~15u;
    // ql: bytes [64h, 64h+64) of the block: 5 lines from b16 + 64h
    uint32_t w[20];
#pragma unroll
    for (int i = 0; i < 5; i++) {
        const uint4 v = lds128(b16 + 64 * h + 16 * i);
        w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
    }
#pragma unroll
    for (int i = 0; i < 16; i++) ql[i] = __funnelshift_r(w[WO + i], w[WO + i + 1], sh);
    // qh: bytes [128 + 32h, +32): 3 lines
    uint32_t u[12];
#pragma unroll
    for (int i = 0; i < 3; i++) {
        const uint4 v = lds128(b16 + 128 + 32 * h + 16 * i);
        u[4 * i] = v.x; u[4 * i + 1] = v.y; u[4 * i + 2] = v.z; u[4 * i + 3] = v.w;
    }
#pragma unroll
    for (int i = 0; i < 8; i++) qh[i] = __funnelshift_r(u[WO + i], u[WO + i + 1], sh);
    // the half's 8 scales at 192 + 8h and d at 208
    const uint4 v = lds128(b16 + 192);
    const uint4 v2 = lds128(b16 + 208);
    const uint32_t t[8] = {v.x, v.y, v.z, v.w, v2.x, v2.y, v2.z, v2.w};
    sc01 = __funnelshift_r(t[WO + 2 * h], t[WO + 2 * h + 1], sh);
    sc23 = __funnelshift_r(t[WO + 2 * h + 1], t[WO + 2 * h + 2], sh);
    dh = __funnelshift_r(t[WO + 4], t[WO + 5], sh) & 0xFFFFu;
}

// One slice of the lane's Q6_K row.  Lane half h takes the block's half h:
// elements 128h + l + 32q (l = 0..31, q = 0..3) with scales sc[8h + l/16 + 2q].
template <int NR>
__device__ __forceinline__ bool q6k_slice(uint32_t base, int kbn, int kb0, const A8Params &p, const ActSmem &as,
                                          float (&tot)[NR], uint32_t rec) {
    const int h = threadIdx.x & 1;
    bool bad = false;
#pragma unroll
    for (int bl = 0; bl < kKC; bl++) {
        if (bl >= kbn) break;
        const uint32_t blk = base + bl * 210;
        uint32_t ql[16], qh[8], sc01, sc23, dh;
        switch ((blk >> 2) & 3) {
        case 0: q6k_load<0>(blk, h, ql, qh, sc01, sc23, dh); break;
        case 1: q6k_load<1>(blk, h, ql, qh, sc01, sc23, dh); break;
        case 2: q6k_load<2>(blk, h, ql, qh, sc01, sc23, dh); break;
        default: q6k_load<3>(blk, h, ql, qh, sc01, sc23, dh); break;
        }
        bad |= !f16_finite(dh);
        const float d = f16f(dh);
        // 6-bit quants of the four quarters, 4 per word (quant.go:318-344)
        uint32_t Q[32];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            Q[i] = (ql[i] & 0x0F0F0F0Fu) | ((qh[i] & 0x03030303u) << 4);
            Q[8 + i] = (ql[8 + i] & 0x0F0F0F0Fu) | (((qh[i] >> 2) & 0x03030303u) << 4);
            Q[16 + i] = ((ql[i] >> 4) & 0x0F0F0F0Fu) | (((qh[i] >> 4) & 0x03030303u) << 4);
            Q[24 + i] = ((ql[8 + i] >> 4) & 0x0F0F0F0Fu) | (((qh[i] >> 6) & 0x03030303u) << 4);
        }
        const int kb = kb0 + bl;
#pragma unroll
        for (int a = 0; a < NR; a++) {
            if (a >= p.rows) break;
            const uint32_t ya = as.q + (uint32_t)(a * p.K + kb * 256 + 128 * h);
            const uint4 ysv = lds128(as.ys + (uint32_t)((a * p.K / 16 + kb * 16 + 8 * h) * 2));
            const uint32_t ysw[4] = {ysv.x, ysv.y, ysv.z, ysv.w};
            int S = 0;
#pragma unroll
            for (int qq = 0; qq < 4; qq++) {
#pragma unroll
                for (int lh = 0; lh < 2; lh++) {
                    const uint4 v = lds128(ya + 32 * qq + 16 * lh);
                    int g = 0;
                    g = __dp4a((int)Q[8 * qq + 4 * lh + 0], (int)v.x, g);
                    g = __dp4a((int)Q[8 * qq + 4 * lh + 1], (int)v.y, g);
                    g = __dp4a((int)Q[8 * qq + 4 * lh + 2], (int)v.z, g);
                    g = __dp4a((int)Q[8 * qq + 4 * lh + 3], (int)v.w, g);
                    const int gi = 2 * qq + lh;  // group of 16: ys index and scale index
                    const int ys = (int)(int16_t)((ysw[gi >> 1] >> (16 * (gi & 1))) & 0xFFFF);
                    const int sc = sbyte(gi < 4 ? sc01 : sc23, gi & 3);
                    S += sc * (g - 32 * ys);
                }
            }
            S += __shfl_xor_sync(FULL, S, 1);
            const float dx = __uint_as_float(lds32(as.dx + (uint32_t)((a * p.nb + kb) * 4)));
            const float fs = __int2float_rn(S), pd = __fmul_rn(d, dx);
            if (rec) {
                if (h == 0) sts128(rec + (uint32_t)(((bl * NR + a) * kRowsW) * 16), fs, pd, 0.f, 0.f);
            } else {
                tot[a] = __fmaf_rn(fs, pd, tot[a]);
            }
        }
    }
    return bad;
}

template <int NR>
__global__ void __launch_bounds__(kThreads, 2) gemv_a8_kernel(const __grid_constant__ A8Params p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = (uint64_t *)smem;
    uint64_t *empty = full + kStages;
    int *badw = (int *)(empty + kStages);            // [kWarps] bad-row masks of parts > 0
    uint8_t *actp = smem + kHeader;
    uint8_t *recp = actp + p.act_bytes;               // [kWarps][rec_bytes] per-block values of parts > 0
    uint8_t *tiles = smem + ((kHeader + p.act_bytes + kWarps * p.rec_bytes + 127) & ~127);  // 128-byte aligned
    uint64_t *actbar = (uint64_t *)(smem + 64);      // completion of the activations' bulk copies
    // the segment table also lives in the dynamic header: a static __shared__
    // variable would move the dynamic base off the 128-byte alignment the
    // 2-D TMA destinations need
    SegTable &tab = *(SegTable *)(smem + 128);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = p.split, slots = kWarps / S;
    const int total = p.seg_g0[p.nseg];
    const int rounds = (total - (int)blockIdx.x + (int)gridDim.x * slots - 1) / ((int)gridDim.x * slots);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kWarps);
        }
        mbar_init(actbar, 1);
        fence_barrier_init();
#pragma unroll
        for (int i = 0; i < kMaxSegs; i++) tab.seg[i] = p.seg[i];
#pragma unroll
        for (int i = 0; i <= kMaxSegs; i++) tab.g0[i] = p.seg_g0[i];
        tab.nseg = p.nseg;
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == kWarps) {
        // producer warp: lane w < kWarps fetches consumer warp w's slice of
        // each stage (its group's 16 rows, chunk part*cpp + i); lane 0 owns
        // the barriers.  2-D mode: one tiled TMA box per warp.  1-D mode:
        // lane l copies row l%16 of warp l/16's slice (two passes).
        int it = 0;
        bool ok = true;
        for (int t = 0; t < rounds && ok; t++) {
            for (int i = 0; i < p.cpp && ok; i++, it++) {
                const int s = it % kStages;
                if (it >= kStages) {
                    int okl = 1;
                    if (lane == 0) okl = mbar_wait_bounded(&empty[s], ((it / kStages) - 1) & 1, p.status);
                    ok = __shfl_sync(FULL, okl, 0) != 0;
                    if (!ok) break;
                }
                if (p.tma2d) {
                    const int w = lane;
                    int g = total, c = p.chunks, si = 0;
                    if (w < kWarps) {
                        g = group_of(blockIdx.x, w / S, slots, t);
                        c = (w % S) * p.cpp + i;
                    }
                    const bool act = g < total && c < p.chunks;
                    int bb = 0, bx = 0, r0 = 0;
                    if (act) {
                        si = find_seg(tab, g);
                        bb = block_bytes(tab.seg[si].dt);
                        bx = box_bytes(tab.seg[si].dt);
                        r0 = (g - tab.g0[si]) * kRowsW;
                    }
                    const unsigned bytes = __reduce_add_sync(FULL, act ? (unsigned)(kRowsW * bx) : 0u);
                    if (lane == 0) mbar_arrive_expect_tx(&full[s], bytes);
                    __syncwarp();
                    if (act) {
                        const int xb = (c * kKC * bb) & ~15;  // byte offset of the box in the row
                        uint8_t *dst = tiles + (size_t)s * p.stage_bytes + (size_t)w * kRowsW * kBoxMax;
                        asm volatile(
                            "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
                            "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
                            "l"((const void *)&p.tmap[si]), "r"(xb / 8), "r"(r0), "r"(smem_u32(&full[s]))
                            : "memory");
                    }
                } else {
                    unsigned bytes = 0;
                    uintptr_t lo[2] = {0, 0}, hi[2] = {0, 0};
                    for (int half = 0; half < 2; half++) {
                        const int w = 2 * half + (lane >> 4), r = lane & 15;
                        if (w >= kWarps) continue;
                        const int g = group_of(blockIdx.x, w / S, slots, t);
                        const int c = (w % S) * p.cpp + i;
                        if (g >= total || c >= p.chunks) continue;
                        const int si = find_seg(tab, g);
                        const GemvSeg &sg = tab.seg[si];
                        const int r0 = (g - tab.g0[si]) * kRowsW;
                        if (r >= sg.n - r0) continue;
                        const int bb = block_bytes(sg.dt), kb0 = c * kKC, kbn = min(kKC, p.nb - kb0);
                        const uintptr_t a = (uintptr_t)(sg.w + (long long)(r0 + r) * row_bytes(sg.dt, p.K) +
                                                        (long long)kb0 * bb);
                        lo[half] = a & ~(uintptr_t)15;
                        hi[half] = (a + (uintptr_t)kbn * bb + 15) & ~(uintptr_t)15;
                        bytes += (unsigned)(hi[half] - lo[half]);
                    }
                    bytes = __reduce_add_sync(FULL, bytes);
                    if (lane == 0) mbar_arrive_expect_tx(&full[s], bytes);
                    __syncwarp();
                    for (int half = 0; half < 2; half++)
                        if (hi[half] > lo[half])
                            bulk_g2s(tiles + (size_t)s * p.stage_bytes + (size_t)(32 * half + lane) * p.slot,
                                     (const void *)lo[half], (uint32_t)(hi[half] - lo[half]), &full[s]);
                }
            }
        }
        // wait (bounded) for copies still in flight before the block exits
        if (lane == 0)
            for (int u = max(0, it - kStages); u < it; u++)
                mbar_wait_bounded(&full[u % kStages], (u / kStages) & 1, p.status);
        return;
    }

    // ---------------------------------------------- consumers
    pdl_wait();
    // activations into shared memory: quants, scales, sums of 32 and 16, the
    // per-block flags -- one bulk copy each when aligned, else plain loads
    const int nr = p.rows;
    const long long K = p.K;
    const int qb = nr * (int)K, dxb = nr * p.nb * 4, xsb = nr * (int)(K / 32) * 2, ysb = nr * (int)(K / 16) * 2;
    const int okb = nr * p.nb * 4;
    auto pad = [](int b) { return (b + 15) & ~15; };
    uint8_t *dxp = actp + pad(qb), *xsp = dxp + pad(dxb), *ysp = xsp + pad(xsb), *okp = ysp + pad(ysb);
    if (p.act_bulk) {
        if (threadIdx.x == 0) {
            mbar_arrive_expect_tx(actbar, (uint32_t)(pad(qb) + pad(dxb) + pad(xsb) + pad(ysb) + pad(okb)));
            bulk_g2s(actp, p.act.q, (uint32_t)pad(qb), actbar);
            bulk_g2s(dxp, p.act.dx, (uint32_t)pad(dxb), actbar);
            bulk_g2s(xsp, p.act.xs, (uint32_t)pad(xsb), actbar);
            bulk_g2s(ysp, p.act.ys, (uint32_t)pad(ysb), actbar);
            bulk_g2s(okp, p.act.ok, (uint32_t)pad(okb), actbar);
        }
        mbar_wait_bounded(actbar, 0, p.status);
    } else {
        const int tid = threadIdx.x;
        for (int i = tid * 16; i < qb; i += kWarps * 32 * 16)
            *(uint4 *)(actp + i) = __ldg((const uint4 *)((const uint8_t *)p.act.q + i));
        for (int i = tid; i < dxb / 4; i += kWarps * 32) ((float *)dxp)[i] = __ldg(p.act.dx + i);
        for (int i = tid; i < xsb / 2; i += kWarps * 32) ((int16_t *)xsp)[i] = __ldg(p.act.xs + i);
        for (int i = tid; i < ysb / 2; i += kWarps * 32) ((int16_t *)ysp)[i] = __ldg(p.act.ys + i);
        for (int i = tid; i < okb / 4; i += kWarps * 32) ((int *)okp)[i] = __ldg(p.act.ok + i);
        asm volatile("bar.sync 1, %0;" ::"r"(kWarps * 32) : "memory");
    }
    ActSmem as;
    as.q = smem_u32(actp);
    as.dx = smem_u32(dxp);
    as.xs = smem_u32(xsp);
    as.ys = smem_u32(ysp);
    // a row is quantized when every one of its blocks is (q8.go:50-97)
    bool act_ok[NR];
#pragma unroll
    for (int a = 0; a < NR; a++) {
        int bad = 0;
        if (a < nr)
            for (int b = lane; b < p.nb; b += 32) bad |= ((const int *)okp)[a * p.nb + b] == 0;
        act_ok[a] = !__any_sync(FULL, bad);
    }

    const int gi = warp / S, part = warp % S;
    const int rlocal = lane >> 1;  // row of this lane within the group's 16
    const uint32_t tiles_s = smem_u32(tiles);
    const uint32_t rec0 = smem_u32(recp) + (uint32_t)(warp * p.rec_bytes) + (uint32_t)(rlocal * 16);
    int it = 0;
    bool failed = false;  // a stage never arrived: skip the work, keep the barrier protocol
    for (int t = 0; t < rounds; t++) {
        const int g = group_of(blockIdx.x, gi, slots, t);
        const bool has = g < total;
        int si = 0, r0 = 0, nrow = 0;
        long long rb = 0;
        if (has) {
            si = find_seg(tab, g);
            r0 = (g - tab.g0[si]) * kRowsW;
            nrow = min(kRowsW, tab.seg[si].n - r0);
            rb = row_bytes(tab.seg[si].dt, K);
        }
        const GemvSeg &sg = tab.seg[si];
        const bool valid = has && rlocal < nrow;
        // the epilogue's bias and residual, requested now so that they are
        // in registers when the products are
        float biasv = 0.f, resv[NR];
#pragma unroll
        for (int a = 0; a < NR; a++) resv[a] = 0.f;
        if (valid && part == 0) {
            if (sg.bias) biasv = sg.bias[r0 + rlocal];
            if (sg.res)
#pragma unroll
                for (int a = 0; a < NR; a++)
                    if (a < nr) resv[a] = sg.res[(long long)a * sg.ldy + r0 + rlocal];
        }
        float tot[NR], off[NR];
#pragma unroll
        for (int a = 0; a < NR; a++) tot[a] = off[a] = 0.f;
        bool bad = false;
        for (int i = 0; i < p.cpp; i++, it++) {
            const int s = it % kStages;
            if (!failed && !mbar_wait_bounded(&full[s], (it / kStages) & 1, p.status)) failed = true;
            const int c = part * p.cpp + i;
            if (has && c < p.chunks && !failed) {
                const int kb0 = c * kKC, kbn = min(kKC, p.nb - kb0);
                const int rr = min(rlocal, nrow - 1);
                // its 16-byte phase: where the slice starts within the staged bytes
                const uintptr_t src = (uintptr_t)(sg.w + (long long)(r0 + rr) * rb + (long long)kb0 * block_bytes(sg.dt));
                const uint32_t row_off = p.tma2d ? (uint32_t)(warp * kRowsW * kBoxMax + rr * box_bytes(sg.dt))
                                                 : (uint32_t)((warp * kRowsW + rr) * p.slot);
                const uint32_t base = tiles_s + (uint32_t)(s * p.stage_bytes) + row_off + (uint32_t)(src & 15);
                // parts > 0 record their per-block values for part 0's chain
                const uint32_t rec = part ? rec0 + (uint32_t)(i * kKC * NR * kRowsW * 16) : 0u;
                if (sg.dt == Q4_K)
                    bad |= q4k_slice<NR>(base, kbn, kb0, p, as, tot, off, rec);
                else
                    bad |= q6k_slice<NR>(base, kbn, kb0, p, as, tot, rec);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        // rows with a refused block scale, from every part of the group
        unsigned badrows = __ballot_sync(FULL, valid && bad);
        if (S > 1) {
            if (part && lane == 0) badw[warp] = (int)badrows;
            asm volatile("bar.sync %0, %1;" ::"r"(2 + gi), "r"(S * 32) : "memory");
            if (part == 0) {
                for (int q = 1; q < S; q++) badrows |= (unsigned)badw[warp + q];
                // continue the block-ordered chain through parts 1..S-1
                for (int q = 1; q < S; q++) {
                    const int nblk = min(p.cpp * kKC, p.nb - q * p.cpp * kKC);
                    const uint32_t rq = rec0 + (uint32_t)(q * p.rec_bytes);
                    for (int j = 0; j < nblk; j++) {
#pragma unroll
                        for (int a = 0; a < NR; a++) {
                            if (a >= nr) break;
                            const uint4 v = lds128(rq + (uint32_t)(((j * NR + a) * kRowsW) * 16));
                            tot[a] = __fmaf_rn(__uint_as_float(v.x), __uint_as_float(v.y), tot[a]);
                            if (sg.dt == Q4_K) off[a] = __fmaf_rn(__uint_as_float(v.z), __uint_as_float(v.w), off[a]);
                        }
                    }
                }
            }
            asm volatile("bar.sync %0, %1;" ::"r"(2 + gi), "r"(S * 32) : "memory");  // records free again
            if (part) continue;
        }
        if (!has || failed) continue;
#pragma unroll
        for (int a = 0; a < NR; a++) {
            if (a >= nr) break;
            if (valid && !(badrows & (1u << (rlocal * 2))) && act_ok[a] && (lane & 1) == 0) {
                float r = __fsub_rn(tot[a], off[a]);
                const int row = r0 + rlocal;
                if (sg.bias) r = __fadd_rn(r, biasv);
                if (sg.res) r = __fadd_rn(resv[a], r);
                sg.y[(long long)a * sg.ldy + row] = r;
                for (int q = 0; q < (p.put.N > 1 ? p.put.N : 0); q++)
                    peer_ptr<float>(p.put, q, p.put.off)[p.put.col0 + row] = r;
            }
            // rows whose weights or activations the 8-bit kernel refuses: f32 product
            for (int rr = 0; rr < nrow; rr++) {
                if (act_ok[a] && !(badrows & (1u << (rr * 2)))) continue;
                const int row = r0 + rr;
                float r = row_dot_f32(sg.dt, sg.w + (long long)row * rb, p.x + (long long)a * K, p.nb);
                if (sg.bias) r = __fadd_rn(r, sg.bias[row]);
                if (sg.res) r = __fadd_rn(sg.res[(long long)a * sg.ldy + row], r);
                if (lane == 0) {
                    sg.y[(long long)a * sg.ldy + row] = r;
                    for (int q = 0; q < (p.put.N > 1 ? p.put.N : 0); q++)
                        peer_ptr<float>(p.put, q, p.put.off)[p.put.col0 + row] = r;
                }
            }
        }
    }
    if (p.put.N > 1) {
        // the warp's peer stores are visible system-wide before the kernel
        // ends (the next kernel on this stream publishes the exchange)
        __syncwarp();
        if (lane == 0) __threadfence_system();
    }
}

template <int NR>
cudaError_t prepare_nr() {
    static std::atomic<unsigned long long> done{0};
    return once_per_device(done, [] {
        cudaError_t e =
            cudaFuncSetAttribute(gemv_a8_kernel<NR>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(gemv_a8_kernel<NR>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        return e;
    });
}

template <int NR>
int blocks_per_sm(size_t smem) {
    static size_t key[8] = {0};
    static int val[8] = {0};
    for (int i = 0; i < 8; i++)
        if (key[i] == smem) return val[i];
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_a8_kernel<NR>, kThreads, smem) != cudaSuccess)
        per_sm = 1;
    for (int i = 0; i < 8; i++)
        if (key[i] == 0) {
            key[i] = smem;
            val[i] = per_sm;
            break;
        }
    return per_sm;
}

template <int NR>
cudaError_t launch_nr(A8Params &p, cudaStream_t st, bool pdl) {
    const size_t smem = (size_t)((kHeader + p.act_bytes + kWarps * p.rec_bytes + 127) & ~127) +
                        (size_t)kStages * p.stage_bytes;
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

// cuTensorMapEncodeTiled, fetched from the driver once.
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)ptr;
    });
    return fn;
}

// The 2-D map of a weight matrix: rows of row_bytes as u64 elements, box
// [box_bytes/8, 16 rows], zero fill past either edge.
bool encode_weight_tmap(const GemvSeg &sg, long long rb, CUtensorMap *out) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)(rb / 8), (cuuint64_t)sg.n};
    const cuuint64_t strides[1] = {(cuuint64_t)rb};
    const cuuint32_t box[2] = {(cuuint32_t)(box_bytes(sg.dt) / 8), (cuuint32_t)kRowsW};
    const cuuint32_t estr[2] = {1, 1};
    return fn(out, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, (void *)sg.w, dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The map of a weight matrix, cached per matrix in a host table (cache) or
// encoded afresh on the stack (!cache: nothing is allocated).
bool weight_tmap(const GemvSeg &sg, long long K, CUtensorMap *out, bool cache) {
    const long long rb = row_bytes(sg.dt, K);
    if (rb % 16 || ((uintptr_t)sg.w & 15) || sg.n <= 0) return false;
    if (!cache) return encode_weight_tmap(sg, rb, out);
    static std::mutex mu;
    static std::unordered_map<const void *, std::pair<long long, CUtensorMap>> table;
    std::lock_guard<std::mutex> lk(mu);
    auto it = table.find(sg.w);
    if (it != table.end() && it->second.first == rb * 1000003LL + sg.n) {
        *out = it->second.second;
        return true;
    }
    CUtensorMap m;
    if (!encode_weight_tmap(sg, rb, &m)) return false;
    table[sg.w] = {rb * 1000003LL + sg.n, m};
    *out = m;
    return true;
}

}  // namespace

void *tmap_encode_fn() { return (void *)encode_fn(); }

namespace {

int nr_tpl(int nr) { return nr == 1 ? 1 : nr == 2 ? 2 : nr <= 4 ? 4 : 8; }

int act_bytes_for(int nr, long long K) {
    auto al = [](long long b) { return (b + 15) & ~15LL; };
    return (int)(al(nr * K) + al(nr * (K / 256) * 4) + al(nr * (K / 32) * 2) + al(nr * (K / 16) * 2) +
                 al(nr * (K / 256) * 4));
}

}  // namespace

cudaError_t gemv_a8_prepare() {
    cudaError_t e = prepare_nr<1>();
    if (e == cudaSuccess) e = prepare_nr<2>();
    if (e == cudaSuccess) e = prepare_nr<4>();
    if (e == cudaSuccess) e = prepare_nr<8>();
    if (e == cudaSuccess) e = gemm_a8_tc_prepare();
    if (e == cudaSuccess) e = gemv_row_prepare();
    num_sms();
    return e;
}

cudaError_t launch_gemv_a8(const GemvSeg *segs, int nseg, const float *x, ActQ8 act, int rows, long long K,
                           unsigned *status, cudaStream_t st, bool pdl, bool cache_maps, const P2P *put,
                           const GemvPrefetch *pf, const GemvNorm *nrm, const GemmSplit *split) {
    if (nseg <= 0 || nseg > kMaxSegs || K % 256 != 0 || rows < 0) return cudaErrorInvalidValue;
    if (put && put->N > 1 && (rows != 1 || nseg != 1)) return cudaErrorInvalidValue;  // exchanges carry one row
    if (nrm && rows != 1) return cudaErrorInvalidValue;  // the fused norm makes one row
    if (rows == 0 || K == 0) return cudaSuccess;
    // many activation rows: the tensor-core GEMM (same results bit for bit)
    if ((!put || put->N <= 1) && gemm_a8_tc_ok(segs, nseg, act, rows, K))
        return launch_gemm_a8_tc(segs, nseg, x, act, rows, K, status, st, pdl, split);
    // one activation row: the slab-streaming kernel (same results bit for bit)
    if (rows == 1 && gemv_row_ok(segs, nseg, act, K))
        return launch_gemv_row(segs, nseg, x, act, K, status, st, pdl, put, pf, nrm);
    if (nrm) return cudaErrorInvalidValue;  // the fused norm exists in the one-row kernel only
    A8Params p = {};
    p.nseg = nseg;
    int maxbb = 0, g = 0;
    for (int i = 0; i < nseg; i++) {
        if (segs[i].dt != Q4_K && segs[i].dt != Q6_K) return cudaErrorInvalidValue;
        p.seg[i] = segs[i];
        p.seg_g0[i] = g;
        g += (segs[i].n + kRowsW - 1) / kRowsW;
        maxbb = max(maxbb, block_bytes(segs[i].dt));
    }
    p.seg_g0[nseg] = g;
    if (g == 0) return cudaSuccess;
    p.K = K;
    p.nb = (int)(K / 256);
    p.chunks = (p.nb + kKC - 1) / kKC;
    // row slots: the slice and its 16-byte alignment slack, rounded to 128
    // bytes plus 16, so consecutive rows start 4 banks apart
    p.slot = ((min(kKC, p.nb) * maxbb + 32 + 127) & ~127) + 16;
    // 2-D tiled TMA when every matrix's rows are 16-byte multiples
    p.tma2d = 1;
    for (int i = 0; i < nseg && p.tma2d; i++) p.tma2d = weight_tmap(segs[i], K, &p.tmap[i], cache_maps) ? 1 : 0;
    p.stage_bytes = p.tma2d ? kWarps * kRowsW * kBoxMax : kRowsCta * p.slot;
    // split K across the warps of a CTA when there are too few row groups
    // to give every SM several warps
    p.split = g >= 6 * num_sms() ? 1 : (g >= 2 * num_sms() ? 2 : 4);
    while (p.split > 1 && p.chunks < p.split) p.split >>= 1;
    p.cpp = (p.chunks + p.split - 1) / p.split;
    p.status = status;
    if (put) p.put = *put;
    // activation rows per launch: as many as fit the shared-memory budget
    int per = kMaxNR;
    while (per > 1 && act_bytes_for(per, K) > kActBudget) per >>= 1;
    if (act_bytes_for(1, K) > 96 * 1024) return cudaErrorInvalidValue;
    cudaError_t e = cudaSuccess;
    for (int r0 = 0; r0 < rows && e == cudaSuccess; r0 += per) {
        const int nr = min(per, rows - r0);
        A8Params q = p;
        q.rows = nr;
        q.act_bytes = act_bytes_for(nr, K);
        q.rec_bytes = q.split > 1 ? q.cpp * kKC * nr_tpl(nr) * kRowsW * 16 : 0;
        q.x = x + (long long)r0 * K;
        q.act.q = act.q + (long long)r0 * K;
        q.act.dx = act.dx + (long long)r0 * (K / 256);
        q.act.xs = act.xs + (long long)r0 * (K / 32);
        q.act.ys = act.ys + (long long)r0 * (K / 16);
        q.act.ok = act.ok + (long long)r0 * (K / 256);
        // bulk copies need 16-byte aligned sources; the ActQ8 carving pads
        // every array to 256 bytes, so reading up to the next 16 is in bounds
        auto a16 = [](const void *ptr) { return ((uintptr_t)ptr & 15) == 0; };
        q.act_bulk = a16(q.act.q) && a16(q.act.dx) && a16(q.act.xs) && a16(q.act.ys) && a16(q.act.ok);
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
