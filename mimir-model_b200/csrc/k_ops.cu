// k_ops.cu -- per-token operators of the llama decode step on sm_100a.
//
// References (gsoultan/mimir-model):
//   rms_norm   interp/fast.go:434-485   float64 sum of squares, mean rounded
//              to f32, inv = f32(1/sqrt(mean + eps)), y = (x*inv)*scale with
//              two f32 roundings.
//   rope       interp/fast.go:507-557   cos/sin of pos*inv_freq in float64,
//              rounded to f32; y1 = x1*c - x2*s, y2 = x2*c + x1*s unfused.
//   swiglu     internal/kernels/attn.go:59-73: siluMulF32AVX2 on the first
//              n&~7 elements, float64 on the rest.
//   attention  interp/fast.go:569-751, internal/kernels/attn.go:26-121 and
//              attn_amd64.s: the vector path of rows without masked holes,
//              the scalar path otherwise; f16 keys and values converted
//              exactly.
//   argmax     cmd/mim-run/main.go:184-193: first index of the maximum
//              (0 when v[0] is NaN), as a 64-bit key reduced by atomicMax.
#include <algorithm>
#include <cfloat>

#include "amd64_math.cuh"
#include "common.cuh"
#include "kernels.h"
#include "p2p.cuh"
#include "rms.cuh"

namespace mimgpu {

namespace {

cudaLaunchConfig_t make_cfg(dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl, cudaLaunchAttribute *attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cfg;
}

__global__ void __launch_bounds__(256) rmsnorm_kernel(const float *__restrict__ x, int n, const float *__restrict__ scale,
                                                      float eps, float *__restrict__ y) {
    __shared__ double dred[8];
    pdl_launch_dependents();
    pdl_wait();
    const int row = blockIdx.x, t = threadIdx.x;
    const float *xr = x + (long long)row * n;
    double ss = 0;
    for (int i = t; i < n; i += 256) {
        const double e = (double)xr[i];
        ss = __fma_rn(e, e, ss);
    }
    ss = warp_sum_d(ss);
    if ((t & 31) == 0) dred[t >> 5] = ss;
    __syncthreads();
    double tot = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) tot += dred[i];
    // the reference's in-order sum where the tree sum cannot settle f32(ss/n)
    float ms;
    if (!rms_mean_certain(tot, n, n / 256 + 16, ms)) {
        __shared__ float ms_seq;
        if (t == 0) ms_seq = (float)__ddiv_rn(rms_seq_sum(xr, n), (double)n);
        __syncthreads();
        ms = ms_seq;
    }
    const float inv = rms_inv_of_mean(ms, eps);
    for (int i = t; i < n; i += 256) {
        float v = __fmul_rn(xr[i], inv);
        if (scale) v = __fmul_rn(v, scale[i]);
        y[(long long)row * n + i] = v;
    }
}

// One block per (b, t); threads over heads x pairs.
__global__ void rope_kernel(const float *__restrict__ x, int H, int T, int D, const int64_t *__restrict__ pos,
                            int pos_rows, const double *__restrict__ inv_freq, int rotary, int interleaved,
                            float *__restrict__ y) {
    extern __shared__ float cs[];  // 2 * rotary/2
    pdl_launch_dependents();
    pdl_wait();
    const int bt = blockIdx.x, b = bt / T, t = bt % T, h = rotary / 2;
    const double pp = (double)pos[(pos_rows != 1 ? b : 0) * T + t];
    for (int i = threadIdx.x; i < h; i += blockDim.x) {
        const double ang = __dmul_rn(pp, inv_freq[i]);
        double s, c;
        sincos(ang, &s, &c);
        cs[2 * i] = (float)c;
        cs[2 * i + 1] = (float)s;
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < H * D; idx += blockDim.x) {
        const int hd = idx / D, e = idx % D;
        const long long at = (((long long)b * H + hd) * T + t) * D;
        float out;
        if (e >= rotary) {
            out = x[at + e];
        } else {
            int i, first;
            if (interleaved) { i = e >> 1; first = !(e & 1); }
            else { i = e < h ? e : e - h; first = e < h; }
            const int i1 = interleaved ? 2 * i : i, i2 = interleaved ? 2 * i + 1 : i + h;
            const float x1 = x[at + i1], x2 = x[at + i2], c = cs[2 * i], s = cs[2 * i + 1];
            out = first ? __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s)) : __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
        }
        y[at + e] = out;
    }
}


__global__ void swiglu_kernel(const float *__restrict__ a, const float *__restrict__ b, long long n, float *__restrict__ y) {
    pdl_launch_dependents();
    pdl_wait();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        y[i] = i < (n & ~7LL) ? silu_mul_amd64(a[i], b[i]) : silu_mul_f64(a[i], b[i]);
}

__global__ void add_kernel(const float *__restrict__ a, const float *__restrict__ b, long long n, float *__restrict__ y) {
    pdl_launch_dependents();
    pdl_wait();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        y[i] = __fadd_rn(a[i], b[i]);
}

__global__ void cast_f16_kernel(const float *__restrict__ x, uint16_t *__restrict__ y, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        y[i] = f32_to_f16(x[i]);
}

__device__ __forceinline__ float kv_at(const void *base, int f16, long long i) {
    return f16 ? f16_to_f32(((const uint16_t *)base)[i]) : ((const float *)base)[i];
}

// ---------------------------------------------------------- attention (general)
// One 256-thread block per query row (b, h, i); scores in dynamic shared memory.
// Rows whose visible keys [st, end) hold no masked key take the reference's
// vector path (attendRow, interp/fast.go:728-751, with the amd64 kernels:
// 8 fused lanes per score in the group-of-four / tail orders, Cephes expf on
// the first n&~7 keys with the lane-sum order, fused key-ordered weighted
// sum); rows with holes, or whose largest score is not finite, take the
// scalar path of fast.go:661-716 (dotF32Go scores, masked keys -inf, exp in
// float64, sequential sum, unfused accumulation skipping zero weights).
__global__ void __launch_bounds__(256) attention_kernel(const AttnArgs a) {
    extern __shared__ float sc[];
    __shared__ float red[8];
    __shared__ int ired[8];
    __shared__ float qsh[512];
    __shared__ float lsum[8], ssum;
    const int t = threadIdx.x, lane = t & 31, w = t >> 5;
    const int row = blockIdx.x;
    const int i = row % a.Tq, h = (row / a.Tq) % a.Hq, b = row / (a.Tq * a.Hq);
    const int G = a.Hq / a.Hkv, kvh = b * a.Hkv + h / G, D = a.D;
    const float *q = a.q + (long long)row * D;
    for (int d = t; d < D; d += 256) qsh[d] = q[d];
    const long long kvoff = (long long)kvh * a.Tk * D;
    const uint8_t *mrow = a.mask ? a.mask + b * a.mst[0] + h * a.mst[1] + i * a.mst[2] : nullptr;
    const bool in_order = !a.mask || a.mst[3] == 1;
    // visible range [st, end) of a boolean mask row, interp/fast.go:606-636
    int end = a.Tk, st = 0;
    if (a.mask && in_order) {
        int last = -1, first = a.Tk;
        for (int j = t; j < a.Tk; j += 256)
            if (mrow[j]) { last = max(last, j); first = min(first, j); }
        for (int o = 16; o; o >>= 1) {
            last = max(last, __shfl_xor_sync(0xffffffffu, last, o));
            first = min(first, __shfl_xor_sync(0xffffffffu, first, o));
        }
        if (lane == 0) { ired[w] = last; red[w] = __int_as_float(first); }
        __syncthreads();
        last = -1; first = a.Tk;
        for (int k = 0; k < 8; k++) { last = max(last, ired[k]); first = min(first, __float_as_int(red[k])); }
        __syncthreads();
        end = last + 1;
        st = first < end ? first : end;
    }
    if (a.causal) end = max(0, min(end, i + (a.Tk - a.Tq) + 1));
    __syncthreads();
    bool vector_path = in_order && st < end;
    if (vector_path && a.mask) {
        int hole = 0;
        for (int j = st + t; j < end; j += 256) hole |= mrow[j] == 0;
        vector_path = !__syncthreads_or(hole);
    }
    float mx;
    int n, j0;
    if (vector_path) {
        // scores of keys st.. as scoresF16AVX2 / scoresF32AVX2
        j0 = st;
        n = end - st;
        const int l = t & 7, grp = t >> 3, n4 = n & ~3;
        for (int base = 0; base < n; base += 32) {
            const int j = base + grp;
            float acc = 0.f;
            if (j < n) {
                const long long kr = kvoff + (long long)(j0 + j) * D;
                for (int c = 0; c < D / 8; c++) acc = __fmaf_rn(qsh[8 * c + l], kv_at(a.k, a.kv_f16, kr + 8 * c + l), acc);
            }
            const float v = score_combine(acc, j >= n4);
            if (j < n && l == 0) sc[j] = __fmul_rn(v, a.scale);
        }
        __syncthreads();
        float m = -INFINITY;
        int nan = 0;
        for (int j = t; j < n; j += 256) {
            const float s = sc[j];
            if (s != s) nan = 1; else m = fmaxf(m, s);
        }
        m = warp_max(m);
        if (lane == 0) red[w] = m;
        nan = __syncthreads_or(nan);
        mx = red[0];
        for (int k = 1; k < 8; k++) mx = fmaxf(mx, red[k]);
        __syncthreads();
        vector_path = !nan && mx != INFINITY && mx != -INFINITY;
    }
    if (!vector_path) {
        // scalar scores of keys 0..end: dotF32Go's four strided lanes, then
        // times scale plus zero; masked keys -inf
        j0 = 0;
        n = end;
        const int l = t & 3, grp = t >> 2, D4 = D & ~3;
        for (int base = 0; base < n; base += 64) {
            const int j = base + grp;
            float acc = 0.f;
            if (j < n) {
                const long long kr = kvoff + (long long)j * D;
                for (int e = l; e < D4; e += 4) acc = __fadd_rn(acc, __fmul_rn(qsh[e], kv_at(a.k, a.kv_f16, kr + e)));
                if (l == 0)
                    for (int e = D4; e < D; e++) acc = __fadd_rn(acc, __fmul_rn(qsh[e], kv_at(a.k, a.kv_f16, kr + e)));
            }
            const float a1 = __shfl_xor_sync(0xffffffffu, acc, 1);    // s0+s1 / s2+s3
            const float p = __fadd_rn((l & 1) ? a1 : acc, (l & 1) ? acc : a1);
            const float p2 = __shfl_xor_sync(0xffffffffu, p, 2);
            const float tot = __fadd_rn((l & 2) ? p2 : p, (l & 2) ? p : p2);
            if (j < n && l == 0) {
                bool allowed = !a.causal || j <= i + (a.Tk - a.Tq);
                if (a.mask) allowed = allowed && mrow[(long long)j * a.mst[3]] != 0;
                sc[j] = allowed ? __fadd_rn(__fmul_rn(tot, a.scale), 0.f) : -INFINITY;
            }
        }
        __syncthreads();
        float m = -INFINITY;
        int nan = 0;
        for (int j = t; j < n; j += 256) {
            const float s = sc[j];
            if (s != s) nan = 1; else m = fmaxf(m, s);
        }
        m = warp_max(m);
        if (lane == 0) red[w] = m;
        nan = __syncthreads_or(nan);
        mx = red[0];
        for (int k = 1; k < 8; k++) mx = fmaxf(mx, red[k]);
        if (nan) mx = __int_as_float(0x7fc00000);
        __syncthreads();
    }
    if (vector_path) {
        const int n8 = n >= 8 ? (n & ~7) : 0;
        for (int j = t; j < n; j += 256) {
            const float x = __fsub_rn(sc[j], mx);
            sc[j] = j < n8 ? expf_amd64(x) : (float)exp((double)x);
        }
        __syncthreads();
        if (t < 8) {
            float sl = 0.f;
            for (int j = t; j < n8; j += 8) sl = __fadd_rn(sl, sc[j]);
            lsum[t] = sl;
        }
        __syncthreads();
        if (t == 0) {
            float sum = 0.f;
            if (n8) sum = __fadd_rn(__fadd_rn(__fadd_rn(lsum[0], lsum[4]), __fadd_rn(lsum[1], lsum[5])),
                                    __fadd_rn(__fadd_rn(lsum[2], lsum[6]), __fadd_rn(lsum[3], lsum[7])));
            for (int j = n8; j < n; j++) sum = __fadd_rn(sum, sc[j]);
            ssum = sum;
        }
        __syncthreads();
        for (int d = t; d < D; d += 256) {
            float acc = 0.f;
            for (int j = 0; j < n; j++) acc = __fmaf_rn(sc[j], kv_at(a.v, a.kv_f16, kvoff + (long long)(j0 + j) * D + d), acc);
            a.out[(long long)row * D + d] = __fdiv_rn(acc, ssum);
        }
        return;
    }
    const bool mx_neg_inf = mx == -INFINITY;
    for (int j = t; j < n; j += 256) {
        const float s = sc[j];
        sc[j] = (s == -INFINITY && !mx_neg_inf) ? 0.f : (float)exp((double)__fsub_rn(s, mx));
    }
    __syncthreads();
    if (t == 0) {
        float sum = 0.f;
        for (int j = 0; j < n; j++) sum = __fadd_rn(sum, sc[j]);  // masked keys add +0
        ssum = sum;
    }
    __syncthreads();
    for (int d = t; d < D; d += 256) {
        float acc = 0.f;
        for (int j = 0; j < n; j++) {
            const float e = sc[j];
            if (e == 0.f) continue;
            acc = __fadd_rn(acc, __fmul_rn(e, kv_at(a.v, a.kv_f16, kvoff + (long long)j * D + d)));
        }
        a.out[(long long)row * D + d] = __fdiv_rn(acc, ssum);
    }
}

// The logits v come from the kernel just before, which may still run when
// this one starts (programmatic dependent launch): v is not __restrict__, so
// its loads stay after the dependency wait and off the read-only cache.
__global__ void __launch_bounds__(256) argmax_kernel(const float *v, long long n, long long i0,
                                                     int holds_first, unsigned long long *__restrict__ key,
                                                     long long ldv) {
    __shared__ unsigned long long red[8];
    pdl_launch_dependents();
    pdl_wait();
    v += blockIdx.y * ldv;  // row blockIdx.y of a batched step
    key += blockIdx.y;
    unsigned long long best = 0;  // 0: no candidate (every real key is larger)
    for (long long i = blockIdx.x * 256LL + threadIdx.x; i < n; i += gridDim.x * 256LL) {
        const float x = v[i];
        if (x == x) best = max(best, argmax_key(x, i0 + i));
    }
    // a NaN first logit keeps the reference's best = 0: the all-ones key wins
    if (holds_first && blockIdx.x == 0 && threadIdx.x == 0 && n > 0 && v[0] != v[0]) best = ~0ull;
    for (int o = 16; o; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int k = 1; k < 8; k++) best = max(best, red[k]);
        if (best) atomicMax(key, best);
    }
}

}  // namespace

cudaError_t launch_rmsnorm(const float *x, int rows, int n, const float *scale, float eps, float *y, cudaStream_t st,
                           bool pdl) {
    if (rows <= 0 || n <= 0) return cudaSuccess;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(dim3(rows), dim3(256), 0, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, rmsnorm_kernel, x, n, scale, eps, y);
}

cudaError_t launch_rope(const float *x, int B, int H, int T, int D, const int64_t *pos, int pos_rows,
                        const double *inv_freq, int rotary, int interleaved, float *y, cudaStream_t st, bool pdl) {
    if (B * T <= 0) return cudaSuccess;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(dim3(B * T), dim3(256), sizeof(float) * rotary, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, rope_kernel, x, H, T, D, pos, pos_rows, inv_freq, rotary, interleaved, y);
}

static unsigned grid_for(long long n) {
    long long g = (n + 255) / 256;
    return (unsigned)(g > 148LL * 16 ? 148LL * 16 : (g < 1 ? 1 : g));
}

cudaError_t launch_swiglu(const float *a, const float *b, long long n, float *y, cudaStream_t st, bool pdl) {
    if (n <= 0) return cudaSuccess;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(dim3(grid_for(n)), dim3(256), 0, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, swiglu_kernel, a, b, n, y);
}

cudaError_t launch_add(const float *a, const float *b, long long n, float *y, cudaStream_t st, bool pdl) {
    if (n <= 0) return cudaSuccess;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = make_cfg(dim3(grid_for(n)), dim3(256), 0, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, add_kernel, a, b, n, y);
}

cudaError_t launch_cast_f16(const float *x, uint16_t *y, long long n, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    cast_f16_kernel<<<grid_for(n), 256, 0, st>>>(x, y, n);
    return cudaGetLastError();
}

constexpr int kMaxAttnKeys = 49152;

cudaError_t launch_attention(const AttnArgs &a, cudaStream_t st) {
    const long long rows = (long long)a.B * a.Hq * a.Tq;
    if (rows <= 0) return cudaSuccess;
    if (a.Tk > kMaxAttnKeys || a.D > 512 || a.D % 8) return cudaErrorInvalidValue;
    const size_t smem = sizeof(float) * (size_t)(a.Tk > 0 ? a.Tk : 1);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    attention_kernel<<<(unsigned)rows, 256, smem, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_argmax(const float *v, long long n, long long i0, bool holds_first, unsigned long long *key,
                          cudaStream_t st, bool pdl, int rows, long long ldv) {
    if (rows < 1 || rows > 65535) return cudaErrorInvalidValue;
    cudaLaunchAttribute attr[1];
    const long long blocks = std::min<long long>((n + 1023) / 1024, std::max<long long>(1, 2LL * num_sms() / rows));
    cudaLaunchConfig_t cfg =
        make_cfg(dim3((unsigned)std::max<long long>(1, blocks), rows), dim3(256), 0, st, pdl, attr);
    return cudaLaunchKernelEx(&cfg, argmax_kernel, v, n, i0, (int)holds_first, key, ldv);
}

namespace {
__global__ void wait_value_kernel(const uint32_t *addr, uint32_t value, unsigned *status) {
    const uint64_t t0 = global_ns(), limit = dev_wait_limit(status);
    for (uint32_t i = 0;; i++) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
        if (v == value) return;
        if ((i & 63) == 63) {
            if (global_ns() - t0 > limit) break;
            __nanosleep(256);
        }
    }
    atomicOr(status, (unsigned)DEV_TIMEOUT);
}
}  // namespace

cudaError_t launch_wait_value(const uint32_t *addr, uint32_t value, unsigned *status, cudaStream_t st) {
    wait_value_kernel<<<1, 1, 0, st>>>(addr, value, status);
    return cudaGetLastError();
}

int num_sms() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

}  // namespace mimgpu
