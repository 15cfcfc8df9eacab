// k_synth.cu -- seeded synthetic weights generated on the device, for the
// benchmark configurations (random-init weights from N(0, sigma) quantized
// as Q4_K, Q6_K or Q8_0; norm scales from N(1, 0.02)).
//
// The generator is counter based (a splitmix64-style hash of the seed and
// the element index, then Box-Muller in float64), so any rows can be made
// independently.  The encoders are this project's own: Q8_0 follows ggml's
// reference quantizer (quant.go:208-228 of gsoultan/mimir-model); the
// reference has no Q4_K/Q6_K encoder, so those use a min/max fit whose
// blocks decode under quant.go:274-344.  Not part of the hot path.
#include "common.cuh"
#include "kernels.h"

namespace mimgpu {

namespace {

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ double normal_at(uint64_t seed, uint64_t i) {
    const uint64_t a = mix64(seed ^ mix64(2 * i)), b = mix64(seed ^ mix64(2 * i + 1));
    const double u1 = ((double)(a >> 11) + 1.0) * 0x1p-53;
    const double u2 = (double)(b >> 11) * 0x1p-53;
    return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}

__device__ __forceinline__ float f16r(float f) { return f16_to_f32(f32_to_f16(f)); }
__device__ __forceinline__ int clampi(int v, int lo, int hi) { return v < lo ? lo : v > hi ? hi : v; }

// One thread encodes one block.
// Block b of the output holds elements first + b*be.. of the stream.
__global__ void synth_kernel(int dt, uint64_t seed, long long nblocks, int be, float mean, float sigma,
                             uint8_t *__restrict__ out, long long first) {
    const long long b = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (b >= nblocks) return;
    float x[256];
    for (int i = 0; i < be; i++) x[i] = (float)(mean + sigma * normal_at(seed, (uint64_t)(first + b * be + i)));
    if (dt == F32) {
        ((float *)out)[b] = x[0];
        return;
    }
    if (dt == Q8_0) {
        uint8_t *blk = out + b * 34;
        float amax = 0.f;
        for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(x[i]));
        const float d = __fdiv_rn(amax, 127.f), id = d != 0.f ? __fdiv_rn(1.f, d) : 0.f;
        const uint16_t h = f32_to_f16(d);
        blk[0] = h & 0xFF;
        blk[1] = h >> 8;
        for (int i = 0; i < 32; i++) blk[2 + i] = (uint8_t)(int8_t)roundf(__fmul_rn(x[i], id));
        return;
    }
    if (dt == Q4_K) {
        uint8_t *blk = out + b * 144;
        float step[8], off[8], maxstep = 0.f, maxoff = 0.f;
        for (int j = 0; j < 8; j++) {
            float lo = 0.f, hi = 0.f;
            for (int i = 0; i < 32; i++) { lo = fminf(lo, x[32 * j + i]); hi = fmaxf(hi, x[32 * j + i]); }
            step[j] = __fdiv_rn(__fsub_rn(hi, lo), 15.f);
            off[j] = -lo;
            maxstep = fmaxf(maxstep, step[j]);
            maxoff = fmaxf(maxoff, off[j]);
        }
        const float d = f16r(__fdiv_rn(maxstep, 63.f)), dmin = f16r(__fdiv_rn(maxoff, 63.f));
        int sc[8], m[8];
        for (int j = 0; j < 8; j++) {
            sc[j] = d > 0.f ? clampi((int)lrintf(__fdiv_rn(step[j], d)), 0, 63) : 0;
            m[j] = dmin > 0.f ? clampi((int)lrintf(__fdiv_rn(off[j], dmin)), 0, 63) : 0;
        }
        const uint16_t hd = f32_to_f16(d), hm = f32_to_f16(dmin);
        blk[0] = hd & 0xFF; blk[1] = hd >> 8; blk[2] = hm & 0xFF; blk[3] = hm >> 8;
        for (int j = 0; j < 4; j++) {
            blk[4 + j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
            blk[8 + j] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
            blk[12 + j] = (uint8_t)((sc[j + 4] & 0xF) | ((m[j + 4] & 0xF) << 4));
        }
        for (int c = 0; c < 4; c++)
            for (int l = 0; l < 32; l++) {
                int q2[2];
                for (int hh = 0; hh < 2; hh++) {
                    const int j = 2 * c + hh;
                    const float ds = __fmul_rn(d, (float)sc[j]), dm = __fmul_rn(dmin, (float)m[j]);
                    q2[hh] = ds > 0.f ? clampi((int)lrintf(__fdiv_rn(__fadd_rn(x[32 * j + l], dm), ds)), 0, 15) : 0;
                }
                blk[16 + 32 * c + l] = (uint8_t)(q2[0] | (q2[1] << 4));
            }
        return;
    }
    // Q6_K
    uint8_t *blk = out + b * 210;
    float gs[16], maxs = 0.f;
    for (int g = 0; g < 16; g++) {
        float vmax = 0.f, amax = 0.f;
        for (int i = 0; i < 16; i++) {
            const float v = x[16 * g + i];
            if (fabsf(v) > amax) { amax = fabsf(v); vmax = v; }
        }
        gs[g] = __fdiv_rn(vmax, -32.f);
        maxs = fmaxf(maxs, fabsf(gs[g]));
    }
    const float d = f16r(__fdiv_rn(maxs, 127.f));
    int sc[16];
    for (int g = 0; g < 16; g++) sc[g] = d > 0.f ? clampi((int)lrintf(__fdiv_rn(gs[g], d)), -128, 127) : 0;
    uint8_t q[256];
    for (int g = 0; g < 16; g++) {
        const float ds = __fmul_rn(d, (float)sc[g]);
        for (int i = 0; i < 16; i++)
            q[16 * g + i] = (uint8_t)(ds != 0.f ? clampi((int)lrintf(__fdiv_rn(x[16 * g + i], ds)), -32, 31) + 32 : 32);
    }
    for (int hh = 0; hh < 2; hh++) {
        uint8_t *ql = blk + 64 * hh, *qh = blk + 128 + 32 * hh;
        const uint8_t *y = q + 128 * hh;
        for (int l = 0; l < 32; l++) {
            const uint8_t q1 = y[l], q2 = y[l + 32], q3 = y[l + 64], q4 = y[l + 96];
            ql[l] = (uint8_t)((q1 & 0xF) | ((q3 & 0xF) << 4));
            ql[l + 32] = (uint8_t)((q2 & 0xF) | ((q4 & 0xF) << 4));
            qh[l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
        }
    }
    for (int g = 0; g < 16; g++) blk[192 + g] = (uint8_t)(int8_t)sc[g];
    const uint16_t hd = f32_to_f16(d);
    blk[208] = hd & 0xFF;
    blk[209] = hd >> 8;
}

}  // namespace

cudaError_t launch_synth(int dt, uint64_t seed, long long nelems, float mean, float sigma, uint8_t *out,
                         cudaStream_t st, long long first) {
    const int be = block_elems(dt);
    if (nelems % be || first % be) return cudaErrorInvalidValue;
    const long long nb = nelems / be;
    if (nb == 0) return cudaSuccess;
    const int threads = 128;
    synth_kernel<<<(unsigned)((nb + threads - 1) / threads), threads, 0, st>>>(dt, seed, nb, be, mean, sigma, out,
                                                                               first);
    return cudaGetLastError();
}

}  // namespace mimgpu
