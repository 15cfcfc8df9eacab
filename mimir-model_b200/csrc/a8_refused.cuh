// a8_refused.cuh -- the f32 product the 8-bit kernels fall back to for the
// (weight row, activation row) pairs dequant_matmul_a8 refuses: a weight
// block with a non-finite scale, or an activation row with a block the
// quantizer flagged (linearA8, interp/fast.go:282-379 of gsoultan/mimir-model).
// Shared by the GEMV and the tensor-core GEMM so a pair's result does not
// depend on how many activation rows a launch carries.
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace mimgpu {

// Exact f32 product of one weight row (decoded as quant.go does) with x, for
// rows the 8-bit path refuses.  Warp-collective; its own summation order
// (the reference's f32 kernels are tolerance-bound).
static __device__ __noinline__ float row_dot_f32(int dt, const uint8_t *row, const float *x, int nb) {
    const int lane = threadIdx.x & 31;
    float acc = 0.f;
    for (int b = 0; b < nb; b++) {
        const float *xb = x + (long long)b * 256;
        if (dt == Q4_K) {
            const uint8_t *blk = row + (long long)b * 144;
            const float d = f16_to_f32(blk[0] | (blk[1] << 8)), dmin = f16_to_f32(blk[2] | (blk[3] << 8));
            uint32_t sw[3];
            for (int i = 0; i < 3; i++)
                sw[i] = blk[4 + 4 * i] | (blk[5 + 4 * i] << 8) | (blk[6 + 4 * i] << 16) | ((uint32_t)blk[7 + 4 * i] << 24);
            for (int e = lane; e < 256; e += 32) {
                const int c = e >> 6, hi = (e >> 5) & 1, l = e & 31;
                int sc, m;
                q4k_scale_min(sw, 2 * c + hi, sc, m);
                const int qv = hi ? (blk[16 + 32 * c + l] >> 4) : (blk[16 + 32 * c + l] & 15);
                const float w = __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)qv), __fmul_rn(dmin, (float)m));
                acc = __fmaf_rn(xb[e], w, acc);
            }
        } else {
            const uint8_t *blk = row + (long long)b * 210;
            const float d = f16_to_f32(blk[208] | (blk[209] << 8));
            for (int e = lane; e < 256; e += 32) {
                const int h = e >> 7, r = e & 127, quarter = r >> 5, l = r & 31;
                const uint8_t *ql = blk + 64 * h, *qh = blk + 128 + 32 * h;
                const int lowb = (quarter & 1) ? ql[l + 32] : ql[l];
                const int low = (quarter >> 1) ? (lowb >> 4) : (lowb & 15);
                const int qv = (low | (((qh[l] >> (2 * quarter)) & 3) << 4)) - 32;
                const int sc = (int8_t)blk[192 + 8 * h + (l >> 4) + 2 * quarter];
                acc = __fmaf_rn(xb[e], __fmul_rn(__fmul_rn(d, (float)sc), (float)qv), acc);
            }
        }
    }
    return warp_sum(acc);
}

// The same product with the activation element e given by xf(e) (callers
// whose f32 activation is not stored as a vector, e.g. recomputed from the
// residual).  Warp-collective.
template <class XF>
__device__ __forceinline__ float row_dot_f32_fn(int dt, const uint8_t *row, int nb, XF xf) {
    const int lane = threadIdx.x & 31;
    float acc = 0.f;
    for (int b = 0; b < nb; b++) {
        const uint8_t *blk = row + (long long)b * block_bytes(dt);
        for (int e = lane; e < 256; e += 32) acc = __fmaf_rn(xf(b * 256 + e), decode_elem(dt, blk, e), acc);
    }
    return warp_sum(acc);
}

}  // namespace mimgpu
