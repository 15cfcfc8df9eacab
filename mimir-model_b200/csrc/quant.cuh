// quant.cuh -- quantization of one 256-element activation block by a
// 256-thread CUDA block (QuantizeBlocks, internal/kernels/q8.go:50-97 and
// 237-273 of gsoultan/mimir-model), shared by every kernel that produces
// 8-bit activations.
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace mimgpu {

struct QuantScratch {
    float amax[8];
    int bad[8];
};

// Quantizes the block whose element threadIdx.x is v: amax over the block,
// q = RoundToEven(127*x/amax) as float64 gives it (q8_round_f), dx = amax/127, the sums of each
// run of 32 and of 16 quants, and the block's flag (0 when it holds NaN,
// Inf or |x| > 2^60, which the reference refuses).
__device__ __forceinline__ void quant_block_256(float v, long long row, long long K, int blk, ActQ8 act,
                                                QuantScratch &qs) {
    const int t = threadIdx.x, w = t >> 5, lane = t & 31;
    const float a = fabsf(v);
    const bool bad = !(a <= 0x1p60f);
    const float m = warp_max(bad ? 0.f : a);
    const unsigned anyb = __ballot_sync(0xffffffffu, bad);
    if (lane == 0) {
        qs.amax[w] = m;
        qs.bad[w] = anyb != 0;
    }
    __syncthreads();
    float amax = qs.amax[0];
    int anybad = qs.bad[0];
#pragma unroll
    for (int i = 1; i < 8; i++) {
        amax = fmaxf(amax, qs.amax[i]);
        anybad |= qs.bad[i];
    }
    int q = 0;
    if (amax != 0.f && !anybad) q = q8_round_f(v, amax, __fdiv_rn(127.f, amax));
    act.q[row * K + (long long)blk * 256 + t] = (int8_t)q;
    int s16 = q;
    for (int o = 8; o; o >>= 1) s16 += __shfl_xor_sync(0xffffffffu, s16, o);
    const int s32 = s16 + __shfl_xor_sync(0xffffffffu, s16, 16);
    const long long kb = row * (K / 256) + blk;
    if ((lane & 15) == 0) act.ys[kb * 16 + w * 2 + (lane >> 4)] = (int16_t)s16;
    if (lane == 0) act.xs[kb * 8 + w] = (int16_t)s32;
    if (t == 0) {
        act.dx[kb] = __fdiv_rn(amax, 127.f);
        act.ok[kb] = anybad ? 0 : 1;
    }
}

// The same quantization by one warp: lane l holds elements 8l..8l+7 of
// block kb of the row in v (v is the value the block would pass to
// quant_block_256 element by element); amax, refusal, rounding, the sums of
// runs of 16 (lane pairs) and 32 (quads), dx and the flag are
// quant_block_256's, bit for bit.
__device__ __forceinline__ void quant_block_warp(const float (&v)[8], long long row, long long K, int kb,
                                                 ActQ8 act) {
    const int lane = threadIdx.x & 31;
    float am = 0.f;
    int bad = 0;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const float a = fabsf(v[j]);
        const bool b = !(a <= 0x1p60f);
        bad |= b;
        am = fmaxf(am, b ? 0.f : a);
    }
    am = warp_max(am);
    bad = __any_sync(0xffffffffu, bad);
    const bool quant = am != 0.f && !bad;
    const float r127 = quant ? __fdiv_rn(127.f, am) : 0.f;
    uint32_t qw[2] = {0u, 0u};
    int s8 = 0;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const int q = quant ? q8_round_f(v[j], am, r127) : 0;
        s8 += q;
        qw[j >> 2] |= ((uint32_t)q & 0xFFu) << (8 * (j & 3));
    }
    *(uint2 *)(act.q + row * K + (long long)kb * 256 + lane * 8) = make_uint2(qw[0], qw[1]);
    const int s16 = s8 + __shfl_xor_sync(0xffffffffu, s8, 1);
    const int s32 = s16 + __shfl_xor_sync(0xffffffffu, s16, 2);
    const long long bk = row * (K / 256) + kb;
    if ((lane & 1) == 0) act.ys[bk * 16 + (lane >> 1)] = (int16_t)s16;
    if ((lane & 3) == 0) act.xs[bk * 8 + (lane >> 2)] = (int16_t)s32;
    if (lane == 0) {
        act.dx[bk] = __fdiv_rn(am, 127.f);
        act.ok[bk] = bad ? 0 : 1;
    }
}

}  // namespace mimgpu
