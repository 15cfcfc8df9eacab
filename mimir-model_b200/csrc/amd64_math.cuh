// amd64_math.cuh -- the float32 arithmetic of the reference's amd64 vector
// kernels (internal/kernels/attn_amd64.s of gsoultan/mimir-model), restated
// for the GPU so attention and SwiGLU give the reference's bits.
//
//   expf_amd64      Cephes' expf as expSumF32AVX2 evaluates it (:82-237):
//                   f = RoundToEven(t*log2e), r = t - f*C1 - f*C2 (fused),
//                   a degree-5 polynomial with fused multiply-adds, times 2^f,
//                   0 below the limit.  The constants are the kernel's table.
//   silu_mul_amd64  siluMulF32AVX2 (:465-527): h = exp(-|a|/2),
//                   a/(1+h*h) for a >= 0, (a*h)*h/(1+h*h) below, times b.
//   score orders    scoresF16AVX2 / scoresF32AVX2 (:12-80, :308-385): eight
//                   fused-multiply-add lanes a_l; keys in groups of four
//                   combine ((a0+a1)+(a2+a3))+((a4+a5)+(a6+a7)), the last
//                   n%4 keys ((a0+a4)+(a1+a5))+((a2+a6)+(a3+a7)).
#pragma once

#include "common.cuh"

namespace mimgpu {

__device__ __forceinline__ float expf_amd64(float t) {
    const float lo = __uint_as_float(0xc2aeac4fu), log2e = __uint_as_float(0x3fb8aa3bu);
    const float c1 = __uint_as_float(0x3f318000u), c2 = __uint_as_float(0xb95e8083u);
    const bool valid = t >= lo;
    const float u = t > lo ? t : lo;  // the x86 max: its second operand on NaN or equality
    const float f = rintf(__fmul_rn(u, log2e));
    float r = __fmaf_rn(-f, c1, u);
    r = __fmaf_rn(-f, c2, r);
    const float r2 = __fmul_rn(r, r);
    float p = __uint_as_float(0x39506967u);
    p = __fmaf_rn(r, p, __uint_as_float(0x3ab743ceu));
    p = __fmaf_rn(r, p, __uint_as_float(0x3c088908u));
    p = __fmaf_rn(r, p, __uint_as_float(0x3d2aa9c1u));
    p = __fmaf_rn(r, p, __uint_as_float(0x3e2aaaaau));
    p = __fmaf_rn(r, p, __uint_as_float(0x3f000000u));
    p = __fmaf_rn(r2, p, r);
    p = __fadd_rn(p, 1.0f);
    const float y = __fmul_rn(p, __uint_as_float((uint32_t)((int)f + 127) << 23));
    return valid ? y : 0.0f;
}

__device__ __forceinline__ float silu_mul_amd64(float a, float b) {
    const float t = __fmul_rn(__uint_as_float(__float_as_uint(a) | 0x80000000u), 0.5f);
    const float h = expf_amd64(t);
    const float den = __fadd_rn(__fmul_rn(h, h), 1.0f);
    const float num = a >= 0.0f ? a : __fmul_rn(__fmul_rn(a, h), h);
    return __fmul_rn(__fdiv_rn(num, den), b);
}

// The float64 SiLU of the reference's scalar tail (attn.go:70-72).
__device__ __forceinline__ float silu_mul_f64(float a, float b) {
    const double ad = (double)a;
    return (float)__dmul_rn(__ddiv_rn(ad, __dadd_rn(1.0, exp(-ad))), (double)b);
}

// Combines the 8 lane sums of a key's score held by the 8 consecutive lanes
// of an aligned group (lane & 7 = l), in the order of a key inside a group of
// four (tail = false) or of a tail key.  Every lane of the group gets the sum.
__device__ __forceinline__ float score_combine(float a, bool tail) {
    const int lane = threadIdx.x & 31;
    const int o1 = tail ? 4 : 1, o2 = tail ? 1 : 2, o3 = tail ? 2 : 4;
    a = __fadd_rn(a, __shfl_sync(0xffffffffu, a, lane ^ o1));
    a = __fadd_rn(a, __shfl_sync(0xffffffffu, a, lane ^ o2));
    a = __fadd_rn(a, __shfl_sync(0xffffffffu, a, lane ^ o3));
    return a;
}

__device__ __forceinline__ float h2f_bits(uint32_t h) {  // f16 bits -> f32 (exact)
    float f;
    asm("{ .reg .b16 t; mov.b16 t, %1; cvt.f32.f16 %0, t; }" : "=f"(f) : "h"((unsigned short)h));
    return f;
}

}  // namespace mimgpu
