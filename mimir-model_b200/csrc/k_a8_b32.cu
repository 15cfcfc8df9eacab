// k_a8_b32.cu -- dequant_matmul_a8.v1: 8-bit activations in blocks of 32.
//
// Semantics (gsoultan/mimir-model):
//   activations  internal/kernels/q8.go:50-97 (QuantizeBlocks with block 32):
//                per run of 32, d = amax/127, q = RoundToEven(127x/amax) in
//                float64, xs = the run's quant sum, dbs = f32(d * xs).
//   row dot      RowDot.DotQ8, q8.go:143-151: the AVX2 kernels dotQ4KQ8AVX2,
//                dotQ6KQ8AVX2 and dotQ8_0Q8AVX2 (internal/kernels/
//                kernels_amd64.s:441, 763, 1007), the only implementation
//                the reference has for blocks of 32, bit for bit.
//   fallbacks    linearA8, interp/fast.go:282-379: an activation row with
//                NaN, Inf or |x| > 2^60, or a weight row with a non-finite
//                block scale, takes the f32 product.
//
// The AVX2 kernels keep 8 f32 lanes per accumulator; lane l of a run of 32
// holds the exact integer sum over its elements 4l..4l+3.  Here one group of
// 8 threads is one (weight row, activation row) pair and thread l is lane l:
// every per-lane fused multiply-add of the assembly happens in the same
// order on the same operands, and the final horizontal sum (HSUM1,
// kernels_amd64.s:408-413: ((v0+v4)+(v1+v5)) + ((v2+v6)+(v3+v7))) is three
// shuffles within the group.  The lane integers come from dp4a: the int8
// products of the assembly (VPMADDUBSW/VPMADDWD) never saturate for these
// operand ranges, so both are the plain integer sums.
//
// Layout: a CTA of 4 warps takes 16 consecutive weight rows (a warp = 4
// groups = 4 rows) and TA activation rows; each group streams its weight
// row once per launch row-tile and reuses each decoded word for the TA
// activation rows.  Weights and activations are read through the read-only
// cache; the activations of a tile are shared by all 16 groups of a CTA.
#include "common.cuh"
#include "kernels.h"
#include "a8_refused.cuh"

namespace mimgpu {

size_t act_q8_b32_bytes(int rows, long long K) {
    size_t n = 0;
    auto add = [&](size_t b) { n += (b + 255) & ~(size_t)255; };
    add((size_t)rows * K);                         // q
    add((size_t)rows * (K / 32) * 4);              // dx, one per run of 32
    add((size_t)rows * (K / 32) * 2);              // xs
    add((size_t)rows * ((K + 255) / 256) * 4);     // ok, one flag per 256 elements
    return n;
}

ActQ8 act_q8_b32_carve(void *base, int rows, long long K) {
    uint8_t *p = (uint8_t *)base;
    auto take = [&](size_t b) { uint8_t *r = p; p += (b + 255) & ~(size_t)255; return r; };
    ActQ8 a;
    a.q = (int8_t *)take((size_t)rows * K);
    a.dx = (float *)take((size_t)rows * (K / 32) * 4);
    a.xs = (int16_t *)take((size_t)rows * (K / 32) * 2);
    a.ys = nullptr;
    a.ok = (int *)take((size_t)rows * ((K + 255) / 256) * 4);
    return a;
}

// Block (row, c) quantizes elements [256c, 256c + 256) of row `row`, one
// warp per run of 32; its flag is 0 when the 256 elements hold NaN, Inf or
// |x| > 2^60 (the reference then refuses the row).
__global__ void __launch_bounds__(256) quantize_a8_b32_kernel(const float *__restrict__ x, long long K, ActQ8 act) {
    __shared__ int bad_of[8];
    const long long row = blockIdx.x;
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long r = (long long)blockIdx.y * 8 + w;  // run of 32
    int bad = 0;
    if (r * 32 < K) {
        const long long i = row * K + r * 32 + lane;
        const float v = x[i];
        const float a = fabsf(v);
        const bool b = !(a <= 0x1p60f);
        const float amax = warp_max(b ? 0.f : a);
        bad = __any_sync(0xffffffffu, b);
        int q = 0;
        if (amax != 0.f && !bad) q = q8_round_f(v, amax, __fdiv_rn(127.f, amax));
        act.q[i] = (int8_t)q;
        int s = q;
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) {
            act.xs[row * (K / 32) + r] = (int16_t)s;
            act.dx[row * (K / 32) + r] = __fdiv_rn(amax, 127.f);
        }
    }
    if (lane == 0) bad_of[w] = bad;
    __syncthreads();
    if (threadIdx.x == 0) {
        int any = 0;
#pragma unroll
        for (int k = 0; k < 8; k++) any |= bad_of[k];
        act.ok[row * gridDim.y + blockIdx.y] = any ? 0 : 1;
    }
}

namespace {

constexpr int kB32Warps = 4;
constexpr int kB32Rows = kB32Warps * 4;  // weight rows per CTA
constexpr unsigned FULLM = 0xffffffffu;

__device__ __forceinline__ uint32_t ldg_u16(const uint8_t *p) { return __ldg((const unsigned short *)p); }
// A 32-bit word at a 2-byte aligned address (Q6_K and Q8_0 blocks are 210
// and 34 bytes long).
__device__ __forceinline__ uint32_t ldg_u32_a2(const uint8_t *p) { return ldg_u16(p) | (ldg_u16(p + 2) << 16); }
__device__ __forceinline__ int ldg_i32(const int8_t *p) { return __ldg((const int *)p); }
__device__ __forceinline__ int byte_of(uint32_t w, int i) { return (int)((w >> (8 * i)) & 0xFFu); }
__device__ __forceinline__ bool f16_inf_nan(uint32_t h) { return (h & 0x7C00u) == 0x7C00u; }

// The f32 product of one weight row with x for a pair the 8-bit kernels
// refuse (warp-collective).
__device__ float refused_dot(int dt, const uint8_t *row, const float *x, long long K) {
    if (dt != Q8_0) return row_dot_f32(dt, row, x, (int)(K / 256));
    const int lane = threadIdx.x & 31;
    float acc = 0.f;
    for (long long e = lane; e < K; e += 32) acc = __fmaf_rn(x[e], decode_elem(Q8_0, row, e), acc);
    return warp_sum(acc);
}

template <int TA>
__global__ void __launch_bounds__(kB32Warps * 32) gemv_a8_b32_kernel(GemvSeg sg, const float *__restrict__ x,
                                                                     ActQ8 act, int rows, long long K) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, t = lane & 7, g = lane >> 3;
    const long long j = (long long)blockIdx.x * kB32Rows + warp * 4 + g;  // this group's weight row
    const long long a0 = (long long)blockIdx.y * TA;
    const int na = (int)min((long long)TA, rows - a0);
    const bool has = j < sg.n;
    const long long rb = row_bytes(sg.dt, K);
    const uint8_t *row = sg.w + (has ? j : 0) * rb;
    const long long K32 = K / 32;
    const int nok = (int)((K + 255) / 256);

    // activation rows the quantizer accepted: every flag of the row set
    bool aok[TA];
#pragma unroll
    for (int a = 0; a < TA; a++) {
        int bad = 0;
        if (a < na)
            for (int b = lane; b < nok; b += 32) bad |= __ldg(act.ok + (a0 + a) * nok + b) == 0;
        aok[a] = a < na && !__any_sync(FULLM, bad);
    }

    float y2[TA], y3[TA];
#pragma unroll
    for (int a = 0; a < TA; a++) y2[a] = y3[a] = 0.f;
    bool wbad = !has;  // a block scale of the row is not finite

    if (sg.dt == Q4_K) {
        // dotQ4KQ8AVX2, kernels_amd64.s:441-562
        const long long nb = K / 256;
        for (long long b = 0; b < nb && !wbad; b++) {
            const uint8_t *blk = row + 144 * b;
            const uint4 hdr = __ldg((const uint4 *)blk);
            if (f16_inf_nan(hdr.x) || f16_inf_nan(hdr.x >> 16)) {
                wbad = true;
                break;
            }
            const float d = f16_to_f32(hdr.x & 0xFFFFu), dmin = f16_to_f32(hdr.x >> 16);
            // get_scale_min_k4 on 32-bit words, as the assembly unpacks them
            const uint32_t sc03 = hdr.y & 0x3f3f3f3fu;
            const uint32_t sc47 = (hdr.w & 0x0f0f0f0fu) | (((hdr.y >> 6) & 0x03030303u) << 4);
            const uint32_t m03 = hdr.z & 0x3f3f3f3fu;
            const uint32_t m47 = ((hdr.w >> 4) & 0x0f0f0f0fu) | (((hdr.z >> 6) & 0x03030303u) << 4);
            const float dm = __fmul_rn(dmin, (float)byte_of(t < 4 ? m03 : m47, t & 3));  // offsets lane = sub-block t
            uint32_t qw[4];
#pragma unroll
            for (int c = 0; c < 4; c++) qw[c] = __ldg((const uint32_t *)(blk + 16 + 32 * c + 4 * t));
#pragma unroll
            for (int a = 0; a < TA; a++) {
                if (!aok[a]) continue;
                const long long ar = a0 + a;
                const int8_t *yq = act.q + ar * K + 256 * b;
                const float *dxp = act.dx + ar * K32 + 8 * b;
                const float4 dA = __ldg((const float4 *)dxp), dB = __ldg((const float4 *)(dxp + 4));
                const float dx[8] = {dA.x, dA.y, dA.z, dA.w, dB.x, dB.y, dB.z, dB.w};
                const float dbs = __fmul_rn(__ldg(dxp + t), (float)__ldg(act.xs + ar * K32 + 8 * b + t));
                y3[a] = __fmaf_rn(dm, dbs, y3[a]);
                float y0 = 0.f, y1 = 0.f;
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    const int slo = __dp4a((int)(qw[c] & 0x0f0f0f0fu), ldg_i32(yq + 64 * c + 4 * t), 0);
                    const int shi = __dp4a((int)((qw[c] >> 4) & 0x0f0f0f0fu), ldg_i32(yq + 64 * c + 32 + 4 * t), 0);
                    const uint32_t scw = c < 2 ? sc03 : sc47;
                    y0 = __fmaf_rn(dx[2 * c], (float)(byte_of(scw, (2 * c) & 3) * slo), y0);
                    y1 = __fmaf_rn(dx[2 * c + 1], (float)(byte_of(scw, (2 * c + 1) & 3) * shi), y1);
                }
                y2[a] = __fmaf_rn(d, __fadd_rn(y0, y1), y2[a]);
            }
        }
    } else if (sg.dt == Q6_K) {
        // dotQ6KQ8AVX2, kernels_amd64.s:763-853
        const long long nb = K / 256;
        const int hi = t >= 4;  // lanes 4..7 take the second scale of a quarter
        for (long long b = 0; b < nb && !wbad; b++) {
            const uint8_t *blk = row + 210 * b;
            const uint32_t dh = ldg_u16(blk + 208);
            if (f16_inf_nan(dh)) {
                wbad = true;
                break;
            }
            const float d = f16_to_f32(dh);
            uint32_t ql[2][2], qh[2], scw[4];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                ql[h][0] = ldg_u32_a2(blk + 64 * h + 4 * t);
                ql[h][1] = ldg_u32_a2(blk + 64 * h + 32 + 4 * t);
                qh[h] = ldg_u32_a2(blk + 128 + 32 * h + 4 * t);
            }
#pragma unroll
            for (int i = 0; i < 4; i++) scw[i] = ldg_u32_a2(blk + 192 + 4 * i);
#pragma unroll
            for (int a = 0; a < TA; a++) {
                if (!aok[a]) continue;
                const long long ar = a0 + a;
                const int8_t *yq = act.q + ar * K + 256 * b;
                const float *dxp = act.dx + ar * K32 + 8 * b;
                const float4 dA = __ldg((const float4 *)dxp), dB = __ldg((const float4 *)(dxp + 4));
                const float dx[8] = {dA.x, dA.y, dA.z, dA.w, dB.x, dB.y, dB.z, dB.w};
                float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
                for (int h = 0; h < 2; h++)
#pragma unroll
                    for (int q = 0; q < 4; q++) {  // quarter: elements 128h + 32q .. +31
                        const uint32_t src = ql[h][q & 1];
                        const uint32_t low = (q >> 1) ? ((src >> 4) & 0x0f0f0f0fu) : (src & 0x0f0f0f0fu);
                        const uint32_t qv = low | (((qh[h] >> (2 * q)) & 0x03030303u) << 4);
                        const int yw = ldg_i32(yq + 128 * h + 32 * q + 4 * t);
                        const int S = __dp4a((int)qv, yw, 0) - 32 * __dp4a(0x01010101, yw, 0);
                        const int sc = (int)(int8_t)byte_of(scw[2 * h + (q >> 1)], 2 * (q & 1) + hi);
                        if (q & 1)
                            acc1 = __fmaf_rn(dx[4 * h + q], (float)(sc * S), acc1);
                        else
                            acc0 = __fmaf_rn(dx[4 * h + q], (float)(sc * S), acc0);
                    }
                y2[a] = __fmaf_rn(d, __fadd_rn(acc0, acc1), y2[a]);
            }
        }
    } else {
        // dotQ8_0Q8AVX2, kernels_amd64.s:1007-1040
        const long long nb = K32;
        for (long long b = 0; b < nb && !wbad; b++) {
            const uint8_t *blk = row + 34 * b;
            const uint32_t dh = ldg_u16(blk);
            if (f16_inf_nan(dh)) {
                wbad = true;
                break;
            }
            const float dw = f16_to_f32(dh);
            const int ww = (int)ldg_u32_a2(blk + 2 + 4 * t);
#pragma unroll
            for (int a = 0; a < TA; a++) {
                if (!aok[a]) continue;
                const long long ar = a0 + a;
                const float scale = __fmul_rn(dw, __ldg(act.dx + ar * K32 + b));
                const int S = __dp4a(ww, ldg_i32(act.q + ar * K + 32 * b + 4 * t), 0);
                y2[a] = __fmaf_rn(scale, (float)S, y2[a]);
            }
        }
    }

    // HSUM1 of Y2 - Y3 within the group, then the bias
#pragma unroll
    for (int a = 0; a < TA; a++) {
        float v = __fsub_rn(y2[a], y3[a]);
        v = __fadd_rn(v, __shfl_xor_sync(FULLM, v, 4));
        v = __fadd_rn(v, __shfl_xor_sync(FULLM, v, 1));
        v = __fadd_rn(v, __shfl_xor_sync(FULLM, v, 2));
        if (t == 0 && !wbad && aok[a]) {
            if (sg.bias) v = __fadd_rn(v, __ldg(sg.bias + j));
            sg.y[(a0 + a) * sg.ldy + j] = v;
        }
    }

    // pairs the 8-bit kernels refuse: the f32 product, one warp per pair
    for (int gg = 0; gg < 4; gg++) {
        const long long jj = (long long)blockIdx.x * kB32Rows + warp * 4 + gg;
        const bool wb = __shfl_sync(FULLM, (int)wbad, 8 * gg) != 0;
        if (jj >= sg.n) continue;
        for (int a = 0; a < na; a++) {
            if (!wb && aok[a]) continue;
            float r = refused_dot(sg.dt, sg.w + jj * rb, x + (a0 + a) * K, K);
            if (sg.bias) r = __fadd_rn(r, __ldg(sg.bias + jj));
            if (lane == 0) sg.y[(a0 + a) * sg.ldy + jj] = r;
        }
    }
}

}  // namespace

bool a8_b32_dtype_ok(int dt, long long K) {
    if (dt == Q8_0) return K > 0 && K % 32 == 0;
    return (dt == Q4_K || dt == Q6_K) && K > 0 && K % 256 == 0;
}

cudaError_t launch_quantize_a8_b32(const float *x, int rows, long long K, ActQ8 act, cudaStream_t st) {
    if (rows <= 0 || K <= 0) return cudaSuccess;
    if (K % 32 || (K + 255) / 256 > 65535) return cudaErrorInvalidValue;
    dim3 grid((unsigned)rows, (unsigned)((K + 255) / 256));
    quantize_a8_b32_kernel<<<grid, 256, 0, st>>>(x, K, act);
    return cudaGetLastError();
}

cudaError_t launch_gemv_a8_b32(const GemvSeg &sg, const float *x, ActQ8 act, int rows, long long K, cudaStream_t st) {
    if (rows <= 0 || sg.n <= 0) return cudaSuccess;
    if (!a8_b32_dtype_ok(sg.dt, K)) return cudaErrorInvalidValue;
    const unsigned gx = (unsigned)((sg.n + kB32Rows - 1) / kB32Rows);
    if (rows == 1) {
        gemv_a8_b32_kernel<1><<<dim3(gx, 1), kB32Warps * 32, 0, st>>>(sg, x, act, 1, K);
        return cudaGetLastError();
    }
    constexpr int TA = 8;
    // grid.y is at most 65535 tiles: larger launches go in pieces
    const long long per = 65535LL * TA;
    for (long long r0 = 0; r0 < rows; r0 += per) {
        const long long nr = rows - r0 < per ? rows - r0 : per;
        GemvSeg s = sg;
        s.y = sg.y + r0 * sg.ldy;
        ActQ8 a = act;
        a.q = act.q + r0 * K;
        a.dx = act.dx + r0 * (K / 32);
        a.xs = act.xs + r0 * (K / 32);
        a.ok = act.ok + r0 * ((K + 255) / 256);
        gemv_a8_b32_kernel<TA><<<dim3(gx, (unsigned)((nr + TA - 1) / TA)), kB32Warps * 32, 0, st>>>(
            s, x + r0 * K, a, (int)nr, K);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace mimgpu
