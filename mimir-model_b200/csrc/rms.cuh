// rms.cuh -- the mean of squares of rms_norm.v1 with the reference's bits.
//
// fastRMSNorm (interp/fast.go:434-485 of gsoultan/mimir-model) sums
// float64(e)^2 over the row IN ORDER, then rounds ss/n to f32:
//     ms  = f32(ss / n)                     (float64 division)
//     inv = f32(1 / sqrt(f64(ms) + f64(f32(eps))))
// A parallel tree sum of the same squares differs from the in-order sum by a
// few float64 ulps, which changes ms only when ss/n lies within that distance
// of an f32 rounding boundary.  Both sums are within (m - 1) u S of the exact
// sum S (u = 2^-53, m = terms summed in sequence; every e^2 is exact in
// float64), so with t the tree sum
//     |ss_seq - t| <= (n + d) u S,   d = the tree's own depth,
// and ss -> f32(ss / n) is monotone: when t - delta and t + delta give the
// same f32 the in-order sum gives it too.  Otherwise (about 2^-15 of rows) one
// thread repeats the reference's in-order sum.
#pragma once

#include "common.cuh"

namespace mimgpu {

// f32(ss / n) for every ss within the tree sum's error bound of `tot`, when
// they agree (returns true and the value in ms).  `depth` bounds the number of
// additions any term went through in the tree.
__device__ __forceinline__ bool rms_mean_certain(double tot, int n, int depth, float &ms) {
    const double delta = __dmul_rn(tot, (double)(2 * (n + depth + 8)) * 0x1p-53);
    const float lo = (float)__ddiv_rn(__dsub_rn(tot, delta), (double)n);
    const float hi = (float)__ddiv_rn(__dadd_rn(tot, delta), (double)n);
    ms = lo;
    return lo == hi;  // false for NaN (non-finite rows take the in-order sum too)
}

// The reference's in-order float64 sum of squares (one thread).
static __device__ __noinline__ double rms_seq_sum(const float *xr, int n) {
    double ss = 0.0;
    for (int i = 0; i < n; i++) {
        const double e = (double)xr[i];
        ss = __fma_rn(e, e, ss);  // e*e is exact in float64: one rounding, as ss += e*e
    }
    return ss;
}

// The same sum over a row other CTAs of the running kernel wrote (read
// through L2, not a possibly stale L1 line).
static __device__ __noinline__ double rms_seq_sum_cg(const float *xr, int n) {
    double ss = 0.0;
    for (int i = 0; i < n; i++) {
        const double e = (double)__ldcg(xr + i);
        ss = __fma_rn(e, e, ss);
    }
    return ss;
}

__device__ __forceinline__ float rms_inv_of_mean(float ms, float eps) {
    return (float)__ddiv_rn(1.0, __dsqrt_rn(__dadd_rn((double)ms, (double)eps)));
}

}  // namespace mimgpu
