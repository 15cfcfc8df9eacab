// gemv_row.cuh -- per-lane block arithmetic of the one-activation-row a8
// products (dequant_matmul_a8.v2, block 256), shared by the stand-alone GEMV
// (k_gemv_row.cu) and the persistent decode step (k_step.cu).
//
// A stage of whole weight rows sits in shared memory; each consumer lane
// takes one half (128 quants) of one 256-element block and computes the exact
// int32 partial sums of dotQ8KRef (internal/kernels/q8k_test.go:35-117 of
// gsoultan/mimir-model): S = sum_s sc_s * sum(q*y) and, for Q4_K,
// M = sum_s m_s * xs_s.  The activation row sits in shared memory in the
// act_off layout with per-half headers (xs of the runs of 32, dx, ok) and the
// sums of 16 (ys) at hdr_off.
#pragma once

#include <cstdint>

#include "common.cuh"

namespace mimgpu {
namespace {

__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ void sts128(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}
__device__ __forceinline__ float f16f(uint32_t h) {  // f16 -> f32 by the hardware conversion (exact)
    float f;
    asm("{ .reg .b16 t; mov.b16 t, %1; cvt.f32.f16 %0, t; }" : "=f"(f) : "h"((unsigned short)h));
    return f;
}
__device__ __forceinline__ int ubyte(uint32_t w, int i) { return (int)((w >> (8 * i)) & 0xFF); }
__device__ __forceinline__ int sbyte(uint32_t w, int i) { return (int)(int8_t)((w >> (8 * i)) & 0xFF); }

// Byte offset of half h of activation block kb.  Rows of 288 bytes (two
// halves of 128 quants + 16 spare), plus 32 bytes every 8 blocks: the
// 16-byte unit of chunk a is 2kb + 2(kb/8) + h + a (mod 8), distinct across
// the 8 lanes of a quarter-warp whether they hold consecutive blocks (Q4_K)
// or blocks 8 apart (Q6_K).
__host__ __device__ __forceinline__ int act_off(int kb, int h) { return kb * 288 + (kb >> 3) * 32 + h * 144; }
__host__ __device__ __forceinline__ int act_bytes(int nb) { return act_off(nb, 0) + 32; }
// Byte offset of the 16-byte per-half entries (headers, sums of 16) of half
// hb = 2kb + h: two spare entries every 16 make the lanes of a quarter-warp
// hit distinct banks in both block orders, as in act_off.
__host__ __device__ __forceinline__ int hdr_off(int hb) { return (hb + ((hb >> 4) << 1)) * 16; }
__host__ __device__ __forceinline__ int hdr_bytes(int nb) { return hdr_off(2 * nb) + 32; }

// Rows [r0, r0 + nr) of an n-row matrix for CTA b of G, cut at multiples of
// u rows (n is one, gemv_row_ok) so that every slab starts on a 16-byte
// boundary and spans a multiple of 16 bytes.
__device__ __forceinline__ void slab(int n, int b, int G, int u, int &r0, int &nr) {
    // n * G < 2^32 (gemv_row_ok): 32-bit quotients
    const unsigned m = (unsigned)(n / u);
    const unsigned a = m * (unsigned)b / (unsigned)G, e = m * (unsigned)(b + 1) / (unsigned)G;
    r0 = (int)a * u;
    nr = (int)(e - a) * u;
}

// The first bytes of slab `sl` of each target launch of pf into L2 (the
// bytes that launch's CTA sl streams first): the launch before it issues this
// for its own CTA's slab once its copies are out.
__device__ __forceinline__ void slab_prefetch(const GemvPrefetch &pf, int sl) {
    for (int t = 0; t < pf.nt; t++) {
        const GemvPrefetchTarget &g = pf.t[t];
        uint32_t left = g.bytes;
        for (int s = 0; s < g.nseg && left; s++) {
            int r0, nr;
            slab(g.n[s], sl, pf.G, g.unit, r0, nr);
            const long long rbn = row_bytes(g.dt[s], g.K);
            const uint8_t *src = g.w[s] + (long long)r0 * rbn;
            long long avail = (long long)nr * rbn;  // a multiple of 16: slabs come in whole units
            while (left && avail > 0) {
                const uint32_t take = (uint32_t)min((long long)min(left, 32768u), avail);
                prefetch_l2(src, take);
                src += take;
                avail -= take;
                left -= take;
            }
        }
    }
}

// The bytes a Q6_K lane needs from one block, read with aligned 16-byte
// loads: WO is the block start's word offset within its 16-byte line
// (warp-uniform), the remaining 0/16-bit shift comes from the address.
template <int WO>
__device__ __forceinline__ void q6k_load(uint32_t blk, int h, uint32_t (&ql)[16], uint32_t (&qh)[8], uint32_t &sc01,
                                         uint32_t &sc23, uint32_t &dh) {
    const uint32_t sh = (blk & 3u) * 8;
    const uint32_t b16 = blk & ~15u;
    uint32_t w[20];
#pragma unroll
    for (int i = 0; i < 5; i++) {
        const uint4 v = lds128(b16 + 64 * h + 16 * i);
        w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
    }
#pragma unroll
    for (int i = 0; i < 16; i++) ql[i] = __funnelshift_r(w[WO + i], w[WO + i + 1], sh);
    uint32_t u[12];
#pragma unroll
    for (int i = 0; i < 3; i++) {
        const uint4 v = lds128(b16 + 128 + 32 * h + 16 * i);
        u[4 * i] = v.x; u[4 * i + 1] = v.y; u[4 * i + 2] = v.z; u[4 * i + 3] = v.w;
    }
#pragma unroll
    for (int i = 0; i < 8; i++) qh[i] = __funnelshift_r(u[WO + i], u[WO + i + 1], sh);
    const uint4 v = lds128(b16 + 192);
    const uint4 v2 = lds128(b16 + 208);
    const uint32_t t[8] = {v.x, v.y, v.z, v.w, v2.x, v2.y, v2.z, v2.w};
    sc01 = __funnelshift_r(t[WO + 2 * h], t[WO + 2 * h + 1], sh);
    sc23 = __funnelshift_r(t[WO + 2 * h + 1], t[WO + 2 * h + 2], sh);
    dh = __funnelshift_r(t[WO + 4], t[WO + 5], sh) & 0xFFFFu;
}

// Half h of a Q4_K block at shared address blk: sub-blocks 4h..4h+3.  The
// exact partial sums S and M of the half, and the block's two scales.
__device__ __forceinline__ void q4k_half(uint32_t blk, int h, uint32_t ya, uint32_t hdr_a, int &S, int &M,
                                         uint32_t &dh, uint32_t &mh, float &dx) {
    const uint4 hdr = lds128(blk);
    uint4 q[4];
#pragma unroll
    for (int i = 0; i < 4; i++) q[i] = lds128(blk + 16 + 64 * h + 16 * i);
    dh = hdr.x & 0xFFFFu;
    mh = hdr.x >> 16;
    // the 4 scales and mins of sub-blocks 4h..4h+3 as packed bytes (getScaleMinK4, quant.go:246-254)
    const uint32_t scw = h ? ((hdr.w & 0x0F0F0F0Fu) | (((hdr.y >> 6) & 0x03030303u) << 4)) : (hdr.y & 0x3F3F3F3Fu);
    const uint32_t mw = h ? (((hdr.w >> 4) & 0x0F0F0F0Fu) | (((hdr.z >> 6) & 0x03030303u) << 4)) : (hdr.z & 0x3F3F3F3Fu);
    const uint32_t qw[16] = {q[0].x, q[0].y, q[0].z, q[0].w, q[1].x, q[1].y, q[1].z, q[1].w,
                             q[2].x, q[2].y, q[2].z, q[2].w, q[3].x, q[3].y, q[3].z, q[3].w};
    // activation chunk a (quants 16a..16a+15 of the half) pairs with the low
    // (a & 2 == 0) or high nibbles of qs chunk 2(a >> 2) + (a & 1)
    int s[4] = {0, 0, 0, 0};
#pragma unroll
    for (int a = 0; a < 8; a++) {
        const uint4 y = lds128(ya + 16 * a);
        const int c = 2 * (a >> 2) + (a & 1), sub = a >> 1;
        const int sh = (a & 2) ? 4 : 0;
        s[sub] = __dp4a((int)((qw[4 * c] >> sh) & 0x0F0F0F0Fu), (int)y.x, s[sub]);
        s[sub] = __dp4a((int)((qw[4 * c + 1] >> sh) & 0x0F0F0F0Fu), (int)y.y, s[sub]);
        s[sub] = __dp4a((int)((qw[4 * c + 2] >> sh) & 0x0F0F0F0Fu), (int)y.z, s[sub]);
        s[sub] = __dp4a((int)((qw[4 * c + 3] >> sh) & 0x0F0F0F0Fu), (int)y.w, s[sub]);
    }
    S = ubyte(scw, 0) * s[0] + ubyte(scw, 1) * s[1] + ubyte(scw, 2) * s[2] + ubyte(scw, 3) * s[3];
    const uint4 ah = lds128(hdr_a);  // xs of the half's 4 runs of 32, dx, ok
    M = ubyte(mw, 0) * (int)(int16_t)(ah.x & 0xFFFF) + ubyte(mw, 1) * (int)(int16_t)(ah.x >> 16) +
        ubyte(mw, 2) * (int)(int16_t)(ah.y & 0xFFFF) + ubyte(mw, 3) * (int)(int16_t)(ah.y >> 16);
    dx = __uint_as_float(ah.z);
}

// Half h of a Q6_K block (elements 128h + l + 32q, scales sc[8h + l/16 + 2q],
// quant.go:318-344): the exact partial sum S.
template <int WO>
__device__ __forceinline__ void q6k_half(uint32_t blk, int h, uint32_t ya, uint32_t ys_a, int &S, uint32_t &dh) {
    uint32_t ql[16], qh[8], sc01, sc23;
    q6k_load<WO>(blk, h, ql, qh, sc01, sc23, dh);
    const uint4 ysv = lds128(ys_a);
    const uint32_t ysw[4] = {ysv.x, ysv.y, ysv.z, ysv.w};
    S = 0;
#pragma unroll
    for (int qq = 0; qq < 4; qq++) {
#pragma unroll
        for (int lh = 0; lh < 2; lh++) {
            const uint4 v = lds128(ya + 32 * qq + 16 * lh);
            const int sh = 2 * qq;
            const uint32_t qs0 = (qq & 1) ? ql[8 + 4 * lh] : ql[4 * lh];
            const uint32_t qs1 = (qq & 1) ? ql[8 + 4 * lh + 1] : ql[4 * lh + 1];
            const uint32_t qs2 = (qq & 1) ? ql[8 + 4 * lh + 2] : ql[4 * lh + 2];
            const uint32_t qs3 = (qq & 1) ? ql[8 + 4 * lh + 3] : ql[4 * lh + 3];
            const int nsh = (qq >> 1) * 4;
            int g = 0;
            g = __dp4a((int)(((qs0 >> nsh) & 0x0F0F0F0Fu) | (((qh[4 * lh] >> sh) & 0x03030303u) << 4)), (int)v.x, g);
            g = __dp4a((int)(((qs1 >> nsh) & 0x0F0F0F0Fu) | (((qh[4 * lh + 1] >> sh) & 0x03030303u) << 4)), (int)v.y, g);
            g = __dp4a((int)(((qs2 >> nsh) & 0x0F0F0F0Fu) | (((qh[4 * lh + 2] >> sh) & 0x03030303u) << 4)), (int)v.z, g);
            g = __dp4a((int)(((qs3 >> nsh) & 0x0F0F0F0Fu) | (((qh[4 * lh + 3] >> sh) & 0x03030303u) << 4)), (int)v.w, g);
            const int gi = 2 * qq + lh;  // group of 16: ys index and scale index
            const int ys = (int)(int16_t)((ysw[gi >> 1] >> (16 * (gi & 1))) & 0xFFFF);
            const int sc = sbyte(gi < 4 ? sc01 : sc23, gi & 3);
            S += sc * (g - 32 * ys);
        }
    }
}

}  // namespace
}  // namespace mimgpu
