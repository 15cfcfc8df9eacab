// common.cuh -- device helpers shared by the sm_100a kernels of libmimgpu.
//
// Bit-exact scalar conversions (float.go:24-88 of gsoultan/mimir-model),
// block-format constants (spec/dtypes.md:124-135), the mbarrier / bulk-copy
// PTX used by the staged GEMV, and bounded waits that report a timeout
// instead of spinning forever.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace mimgpu {

enum DType : int { F32 = 1, F16 = 2, Q8_0 = 64, Q4_K = 66, Q6_K = 67 };

// Error bits a kernel may set in the context's device status word.
enum DevStatus : unsigned { DEV_TIMEOUT = 1u, DEV_BADARG = 2u };

__host__ __device__ inline int block_elems(int dt) {
    return dt == Q4_K || dt == Q6_K ? 256 : dt == Q8_0 ? 32 : 1;
}
__host__ __device__ inline int block_bytes(int dt) {
    return dt == Q4_K ? 144 : dt == Q6_K ? 210 : dt == Q8_0 ? 34 : dt == F16 ? 2 : 4;
}
__host__ __device__ inline long long row_bytes(int dt, long long k) {
    int be = block_elems(dt);
    if (k % be) return 0;
    return k / be * block_bytes(dt);
}

// ---------------------------------------------------------------- f16 bits
// f16 -> f32 exactly, including subnormals, infinities and NaN payloads
// (F16ToF32, float.go:24-43).  Written with integer ops so the NaN payload
// is kept bit for bit.
__device__ __forceinline__ float f16_to_f32(uint32_t h) {
    uint32_t sign = (h & 0x8000u) << 16, exp = (h >> 10) & 0x1Fu, mant = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0x1F) {
        bits = sign | 0x7F800000u | (mant << 13);
    } else if (exp != 0) {
        bits = sign | ((exp + 112u) << 23) | (mant << 13);
    } else if (mant == 0) {
        bits = sign;
    } else {
        // subnormal: mant * 2^-24; normalise with a count of leading zeros
        int lz = __clz(mant) - 21;  // leading zeros within the 11-bit field
        mant = (mant << lz) & 0x3FFu;
        bits = sign | ((uint32_t)(113 - lz) << 23) | (mant << 13);
    }
    return __uint_as_float(bits);
}

// f32 -> f16 with round to nearest even; NaN stays a quiet NaN with the top
// payload bits (F32ToF16, float.go:49-82).
__device__ __forceinline__ uint16_t f32_to_f16(float f) {
    uint32_t b = __float_as_uint(f);
    uint32_t sign = (b >> 16) & 0x8000u;
    int exp = (int)((b >> 23) & 0xFF);
    uint32_t mant = b & 0x7FFFFFu;
    if (exp == 0xFF) return (uint16_t)(mant ? (sign | 0x7E00u | (mant >> 13)) : (sign | 0x7C00u));
    int e = exp - 127 + 15;
    if (e >= 0x1F) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        if (e < -11) return (uint16_t)sign;
        mant |= 0x800000u;
        uint32_t shift = (uint32_t)(14 - e);
        uint32_t half = 1u << (shift - 1);
        uint32_t rem = mant & ((half << 1) - 1);
        uint32_t q = mant >> shift;
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t q = ((uint32_t)e << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
    return (uint16_t)(sign | q);
}

__device__ __forceinline__ bool f16_finite(uint32_t h) { return (h & 0x7C00u) != 0x7C00u; }

// Q4_K sub-block scale and min j (0..7) from the 12 packed bytes
// (getScaleMinK4, quant.go:246-254).  `s` holds the 12 bytes as 3 words.
__device__ __forceinline__ void q4k_scale_min(const uint32_t s[3], int j, int &sc, int &m) {
    // byte i of the 12 packed bytes, selected without a runtime-indexed array
    auto byte = [&](int i) -> int {
        const uint32_t w = i < 4 ? s[0] : (i < 8 ? s[1] : s[2]);
        return (int)((w >> ((i & 3) * 8)) & 0xFFu);
    };
    if (j < 4) {
        sc = byte(j) & 63;
        m = byte(j + 4) & 63;
    } else {
        sc = (byte(j + 4) & 0xF) | ((byte(j - 4) >> 6) << 4);
        m = (byte(j + 4) >> 4) | ((byte(j) >> 6) << 4);
    }
}

// Element i of a row of block-dtype values, decoded exactly as Dequantize
// does (quant.go:197-344).
__device__ __forceinline__ float decode_elem(int dt, const uint8_t *src, long long i) {
    if (dt == Q4_K) {
        const uint8_t *blk = src + (i / 256) * 144;
        const int e = (int)(i % 256), c = e >> 6, hi = (e >> 5) & 1, l = e & 31;
        const float d = f16_to_f32(blk[0] | (blk[1] << 8)), dmin = f16_to_f32(blk[2] | (blk[3] << 8));
        uint32_t sw[3];
        for (int k = 0; k < 3; k++)
            sw[k] = blk[4 + 4 * k] | (blk[5 + 4 * k] << 8) | (blk[6 + 4 * k] << 16) | ((uint32_t)blk[7 + 4 * k] << 24);
        int sc, m;
        q4k_scale_min(sw, 2 * c + hi, sc, m);
        const int q = hi ? (blk[16 + 32 * c + l] >> 4) : (blk[16 + 32 * c + l] & 15);
        return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dmin, (float)m));
    }
    if (dt == Q6_K) {
        const uint8_t *blk = src + (i / 256) * 210;
        const int e = (int)(i % 256), h = e >> 7, r = e & 127, quarter = r >> 5, l = r & 31;
        const float d = f16_to_f32(blk[208] | (blk[209] << 8));
        const uint8_t *ql = blk + 64 * h, *qh = blk + 128 + 32 * h;
        const int lowb = (quarter & 1) ? ql[l + 32] : ql[l];
        const int low = (quarter >> 1) ? (lowb >> 4) : (lowb & 15);
        const int q = (low | (((qh[l] >> (2 * quarter)) & 3) << 4)) - 32;
        const int sc = (int8_t)blk[192 + 8 * h + (l >> 4) + 2 * quarter];
        return __fmul_rn(__fmul_rn(d, (float)sc), (float)q);
    }
    if (dt == Q8_0) {
        const uint8_t *blk = src + (i / 32) * 34;
        return __fmul_rn(f16_to_f32(blk[0] | (blk[1] << 8)), (float)(int8_t)blk[2 + i % 32]);
    }
    if (dt == F16) return f16_to_f32(src[2 * i] | (src[2 * i + 1] << 8));
    return ((const float *)src)[i];
}

// RoundToEven(127 v / amax) for |v| <= amax, 0 < amax < inf, as quantQ8
// (internal/kernels/q8.go:75-86, 251-260 of gsoultan/mimir-model) rounds it:
// the float64 quotient to nearest even, which is the EXACT quotient rounded
// to nearest even (127 v is exact in float64; the float64 quotient is within
// 2^-46 of the exact one, which is a half-integer or at least 2^-34 away from
// one).  Here without a division per element: the estimate t / amax as
// t * inv_a (inv_a = 1.0 / amax, once per block) is at most one off, and only
// next to a half-integer; the remainder t - q amax is exact (both terms have
// at most 31 significant bits, or q = 0) and moves q to the nearest integer,
// ties to the even one.
__device__ __forceinline__ int q8_round(float v, double a, double inv_a) {
    const double t = 127.0 * (double)v;
    double q = rint(__dmul_rn(t, inv_a));
    double r = __fma_rn(-q, a, t);
    const double h = 2.0 * fabs(r);
    if (h > a) q += r > 0.0 ? 1.0 : -1.0;  // then |t - q amax| < amax / 2
    else if (h == a && ((int)q & 1)) q += r > 0.0 ? 1.0 : -1.0;
    return (int)q;
}

// q8_round in float32 where that is provably the same: with r = fl(127/amax)
// and y = fl(v r), |y - 127 v / amax| <= 127 * 2^-23 (< 1.6e-5, plus 2^-149
// when y is subnormal), so when y is farther than 4e-5 from a half-integer
// its nearest integer is the exact quotient's.  Otherwise (about one element
// in 10^4), or for amax below 2^-100 (r could overflow), the exact routine.
// r = __fdiv_rn(127.f, amax), computed once per block.
__device__ __forceinline__ int q8_round_f(float v, float amax, float r) {
    const float y = __fmul_rn(v, r);
    const float f = rintf(y);
    if (fabsf(__fsub_rn(y, f)) < 0.49996f && amax >= 0x1p-100f) return (int)f;
    const double a = (double)amax;
    return q8_round(v, a, __ddiv_rn(1.0, a));
}

// ------------------------------------------------------------- argmax
// argmax (cmd/mim-run/main.go:184-193): best = 0; x > v[best] moves best.
// The result is the first index of the largest non-NaN value (NaNs never
// compare greater), or 0 when v[0] is NaN.  Each block reduces a strided
// share to (value, index) and folds it into one 64-bit key by atomicMax:
// the value's order-preserving bits above the complement of the index, so
// the larger value and then the smaller index wins; -0 counts as +0, as the
// reference's comparison does.  A NaN first value sets the all-ones key.
// With tensor parallelism each rank folds its vocabulary slice (global
// indices i0 + i) and the keys meet in a 64-bit max all-reduce.
__device__ __forceinline__ unsigned long long argmax_key(float v, long long i) {
    uint32_t b = __float_as_uint(v == 0.f ? 0.f : v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)b << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)i);
}

// ------------------------------------------------------- mbarrier / bulk copy
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// The context's limit of one bounded device wait, in nanoseconds: the
// 64-bit word after the status word (mimgpu_set_timeout_ms; 2 s until set).
constexpr uint64_t kDefaultWaitNs = 2000000000ull;
__device__ __forceinline__ uint64_t dev_wait_limit(const unsigned *status) {
    if (!status) return kDefaultWaitNs;
    const uint64_t v = *(volatile const unsigned long long *)(status + 2);
    return v ? v : kDefaultWaitNs;
}

// Waits for the phase with the given parity to complete.  Gives up after the
// context's wait limit (dev_wait_limit) of wall time, sets DEV_TIMEOUT in
// *status and returns false, so a lost arrival ends the kernel with an error
// the host reads instead of a hang.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, unsigned *status) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns(), limit_ns = dev_wait_limit(status);
    for (uint32_t i = 1;; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255) == 0 && global_ns() - t0 > limit_ns) break;
    }
    if (status) atomicOr(status, (unsigned)DEV_TIMEOUT);
    return false;
}

// One-dimensional bulk copy global -> shared, completing on `bar`.  Both
// addresses must be 16-byte aligned and `bytes` a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// The same copy with an L2 eviction policy (createpolicy): evict_first for
// bytes read once, so they do not push out data that is read again.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void bulk_g2s_hint(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                              uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}
// Asynchronous prefetch of `bytes` (a multiple of 16, 16-byte aligned) into L2.
__device__ __forceinline__ void prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void prefetch_l2_hint(const void *src, uint32_t bytes, uint64_t pol) {
    asm volatile("cp.async.bulk.prefetch.L2.global.L2::cache_hint [%0], %1, %2;" ::"l"(src), "r"(bytes), "l"(pol)
                 : "memory");
}

// Loads of small read-only data every step reuses (norm weights, the RoPE
// table) with the L2 evict_last policy, so the weight stream (evict_first)
// does not push them out between steps.
__device__ __forceinline__ float ldg_keep(const float *p, uint64_t pol) {
    float v;
    asm volatile("ld.global.nc.L2::cache_hint.f32 %0, [%1], %2;" : "=f"(v) : "l"(p), "l"(pol));
    return v;
}
__device__ __forceinline__ float2 ldg_keep2(const float2 *p, uint64_t pol) {
    float2 v;
    asm volatile("ld.global.nc.L2::cache_hint.v2.f32 {%0,%1}, [%2], %3;" : "=f"(v.x), "=f"(v.y) : "l"(p), "l"(pol));
    return v;
}
__device__ __forceinline__ float4 ldg_keep4(const float4 *p, uint64_t pol) {
    float4 v;
    asm volatile("ld.global.nc.L2::cache_hint.v4.f32 {%0,%1,%2,%3}, [%4], %5;"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p), "l"(pol));
    return v;
}

// Streaming 128-bit global load that does not allocate in L1.
__device__ __forceinline__ uint4 ldg_stream(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Four bytes starting at a byte address that may be unaligned, read from
// shared memory as two aligned words.
__device__ __forceinline__ uint32_t lds_u32_unaligned(const uint8_t *p) {
    uintptr_t a = (uintptr_t)p;
    const uint32_t *w = (const uint32_t *)(a & ~(uintptr_t)3);
    uint32_t sh = (uint32_t)(a & 3) * 8;
    uint32_t lo = w[0];
    if (sh == 0) return lo;
    return __funnelshift_r(lo, w[1], sh);
}

// Programmatic dependent launch: wait for the grid this one depends on, and
// signal that dependents may start their prologue.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

}  // namespace mimgpu
