// k_gemm_tc.cu -- dequant_matmul_a8.v2 (block 256) for many activation rows
// (prompt processing, batched decode) on the 5th-generation tensor cores.
//
// Same results as the GEMV (k_gemv_a8.cu) and the reference's dotQ8KRef
// (internal/kernels/q8k_test.go:35-117 of gsoultan/mimir-model), bit for
// bit: the exact int32 block sums S (and M for Q4_K), then the block-ordered
// f32 chain tot = fma(float(S), d*dx, tot), off = fma(float(M), dmin*dx, off).
//
// A CTA owns 128 weight rows x 32 activation rows.  For every 256-element
// block it decodes the rows' quants into shared memory as int8 "digit
// planes" whose products with the int8 activations fit the MMA operands
// exactly, and sums each plane over the block with tcgen05.mma kind::i8
// (M 128, N 32, K 32) into TMEM:
//   Q4_K  sc = lo + 8 hi (3-bit digits):  planes q*lo and q*hi in [0, 105],
//         S = A0 + 8 A1 (sub-block scales folded in, per row and sub-block);
//   Q6_K  sc = d0 + 8 d1 + 64 d2 (digits in [-3, 4]): planes (q-32)*d in
//         [-128, 124], S = A0 + 8 A1 + 64 A2.
// The 4 warps read the accumulators back (tcgen05.ld, one row per thread)
// and continue each (row, activation row) chain in registers.  The mins of
// Q4_K, M = sum m_j xs_j, are 8 products on the CUDA cores.
//
// Operands use the K-major canonical layout without swizzle: core matrices
// of 8 rows x 16 bytes (128 contiguous bytes), 8-row groups SBO = 128 bytes
// apart, 16-byte K chunks LBO = rows * 16 bytes apart.
#include <cstdint>

#include "a8_refused.cuh"
#include "common.cuh"
#include "kernels.h"

namespace mimgpu {

namespace {

constexpr int TM = 128;              // weight rows per CTA (MMA M, one TMEM lane each)
constexpr int TN = 32;               // activation rows per CTA (MMA N)
constexpr int kThr = 128;            // 4 warps
constexpr int kPlanes = 3;
constexpr uint32_t kTmemCols = 128;  // 3 planes x 32 columns, rounded to a power of two
constexpr int kRawPitch = 240;       // bytes of one staged raw block row (210 + 16-byte phase, rounded)
constexpr int kPlaneBytes = TM * 256;
constexpr int kBBytes = TN * 256;

struct TcParams {
    GemvSeg seg[kMaxSegs];
    int seg_t0[kMaxSegs + 1];  // first 128-row tile of each segment
    int nseg;
    ActQ8 act;                 // rows x K
    const float *x;            // f32 activations (refused rows)
    int rows;
    long long K;
    int nb;
    unsigned *status;
};

// shared-memory layout (bytes)
constexpr int kOffBar = 0;       // mbarrier of the MMA commits
constexpr int kOffTmem = 16;     // TMEM base address written by tcgen05.alloc
constexpr int kOffMeta = 128;    // per block: dx [TN] f32, ok [TN] i32, xs [TN][8] i16
constexpr int kOffRaw = 1024;
constexpr int kOffPlanes = kOffRaw + TM * kRawPitch;
constexpr int kOffB = kOffPlanes + kPlanes * kPlaneBytes;
constexpr int kSmemTc = kOffB + kBBytes;

// byte offset of (row, k) in a K-major no-swizzle operand of `R` rows x 256
__device__ __forceinline__ uint32_t canon(int row, int k, int R) {
    return (uint32_t)(((k >> 4) * (R >> 3) + (row >> 3)) * 128 + (row & 7) * 16 + (k & 15));
}

__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);  // version 1, no swizzle
}

// kind::i8 instruction descriptor: D s32, A and B signed int8, both K-major,
// N = 32, M = 128
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(TN >> 3) << 17) | ((uint32_t)(TM >> 4) << 24);

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }


// Digits of a Q6_K scale in base 8, each in [-3, 4]: sc = d0 + 8 d1 + 64 d2.
__device__ __forceinline__ void q6_digits(int sc, int &d0, int &d1, int &d2) {
    d0 = ((sc + 3) & 7) - 3;
    int t = (sc - d0) >> 3;
    d1 = ((t + 3) & 7) - 3;
    d2 = (t - d1) >> 3;
}

__global__ void __launch_bounds__(kThr, 1) gemm_a8_tc_kernel(const __grid_constant__ TcParams p) {
    extern __shared__ __align__(1024) uint8_t sm[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint64_t *bar = (uint64_t *)(sm + kOffBar);
    uint32_t *tmem_slot = (uint32_t *)(sm + kOffTmem);
    float *mdx = (float *)(sm + kOffMeta);
    int *mok = (int *)(sm + kOffMeta + 4 * TN);
    int16_t *mxs = (int16_t *)(sm + kOffMeta + 8 * TN);
    uint8_t *raw = sm + kOffRaw;
    uint8_t *planes = sm + kOffPlanes;
    uint8_t *bt = sm + kOffB;

    // the tile: segment, its 128 rows, the 32 activation rows
    const int tile = blockIdx.x;
    int si = 0;
    while (si + 1 < p.nseg && tile >= p.seg_t0[si + 1]) si++;
    GemvSeg sg = p.seg[0];
#pragma unroll
    for (int i = 1; i < kMaxSegs; i++)
        if (i == si) sg = p.seg[i];
    const int r0 = (tile - p.seg_t0[si]) * TM, nrow = min(TM, sg.n - r0);
    const int n0 = blockIdx.y * TN, ntok = min(TN, p.rows - n0);
    const int dt = sg.dt, bb = block_bytes(dt);
    const long long rb = row_bytes(dt, p.K);
    const int P = dt == Q4_K ? 2 : 3;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_barrier_init();
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();
    pdl_wait();

    const int row = tid;                       // this thread's weight row in the tile
    const bool has_row = row < nrow;
    float tot[TN], off[TN];
#pragma unroll
    for (int n = 0; n < TN; n++) tot[n] = off[n] = 0.f;
    bool rowbad = false;
    uint32_t tokbad = 0;                       // activation rows refused (bit n)
    bool failed = false;
    uint32_t phase = 0;
    const uint32_t planes_s = smem_u32(planes), bt_s = smem_u32(bt);

    for (int kb = 0; kb < p.nb; kb++) {
        // ---- raw weight block of every row (16-byte aligned window) -> shared
        {
            const uintptr_t a = has_row ? (uintptr_t)(sg.w + (long long)(r0 + row) * rb + (long long)kb * bb) : 0;
            const uintptr_t lo = a & ~(uintptr_t)15;
            const int nchunk = has_row ? (int)(((a + bb + 15) & ~(uintptr_t)15) - lo) / 16 : 0;
            uint4 *dst = (uint4 *)(raw + row * kRawPitch);
            for (int c = 0; c < nchunk; c++) dst[c] = __ldg((const uint4 *)lo + c);
        }
        // ---- activation block of the 32 rows -> B operand; dx, ok, xs
        for (int id = tid; id < TN * 16; id += kThr) {
            const int n = id >> 4, c = id & 15;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (n < ntok) v = __ldg((const uint4 *)(p.act.q + (long long)(n0 + n) * p.K + (long long)kb * 256 + c * 16));
            *(uint4 *)(bt + canon(n, c * 16, TN)) = v;
        }
        if (tid < TN) {
            const bool in = tid < ntok;
            mdx[tid] = in ? p.act.dx[(long long)(n0 + tid) * p.nb + kb] : 0.f;
            mok[tid] = in ? p.act.ok[(long long)(n0 + tid) * p.nb + kb] : 1;
        }
        for (int id = tid; id < TN * 8; id += kThr) {
            const int n = id >> 3, j = id & 7;
            mxs[id] = n < ntok ? p.act.xs[(long long)(n0 + n) * (p.K / 32) + (long long)kb * 8 + j] : (int16_t)0;
        }
        __syncwarp();  // each thread reads back only its own raw row
        // ---- this row's quants as digit planes in the canonical layout
        const uint8_t *blk = raw + row * kRawPitch +
                             (has_row ? (int)(((uintptr_t)sg.w + (uintptr_t)((r0 + row) * rb) + (uintptr_t)kb * bb) & 15) : 0);
        float d = 0.f, dmin = 0.f;
        int sc8[8] = {0, 0, 0, 0, 0, 0, 0, 0}, mn8[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if (dt == Q4_K) {
            const uint32_t dm = has_row ? (uint32_t)blk[0] | ((uint32_t)blk[1] << 8) | ((uint32_t)blk[2] << 16) |
                                              ((uint32_t)blk[3] << 24)
                                        : 0u;
            rowbad |= has_row && (!f16_finite(dm & 0xFFFFu) || !f16_finite(dm >> 16));
            d = f16_to_f32(dm & 0xFFFFu);
            dmin = f16_to_f32(dm >> 16);
            uint32_t sw[3] = {0, 0, 0};
            if (has_row)
                for (int i = 0; i < 3; i++)
                    sw[i] = blk[4 + 4 * i] | (blk[5 + 4 * i] << 8) | (blk[6 + 4 * i] << 16) | ((uint32_t)blk[7 + 4 * i] << 24);
#pragma unroll
            for (int j = 0; j < 8; j++) q4k_scale_min(sw, j, sc8[j], mn8[j]);
#pragma unroll 4
            for (int ch = 0; ch < 16; ch++) {
                // elements 16ch..16ch+15: sub-block j = ch/2, qs bytes [32c + l0, +16)
                const int j = ch >> 1, c = ch >> 2, hi = (ch >> 1) & 1, l0 = (ch & 1) * 16;
                const int lo3 = sc8[j] & 7, hi3 = sc8[j] >> 3;
                uint32_t w0[4], w1[4];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    uint32_t a0 = 0, a1 = 0;
#pragma unroll
                    for (int v = 0; v < 4; v++) {
                        const int b = has_row ? blk[16 + 32 * c + l0 + 4 * u + v] : 0;
                        const int q = hi ? (b >> 4) : (b & 15);
                        a0 |= (uint32_t)(q * lo3) << (8 * v);
                        a1 |= (uint32_t)(q * hi3) << (8 * v);
                    }
                    w0[u] = a0;
                    w1[u] = a1;
                }
                *(uint4 *)(planes + canon(row, ch * 16, TM)) = make_uint4(w0[0], w0[1], w0[2], w0[3]);
                *(uint4 *)(planes + kPlaneBytes + canon(row, ch * 16, TM)) = make_uint4(w1[0], w1[1], w1[2], w1[3]);
            }
        } else {
            const uint32_t dh = has_row ? (uint32_t)blk[208] | ((uint32_t)blk[209] << 8) : 0u;
            rowbad |= has_row && !f16_finite(dh);
            d = f16_to_f32(dh);
#pragma unroll 2
            for (int ch = 0; ch < 16; ch++) {
                // elements 16ch..16ch+15: half h, quarter qq, l in [l0, l0 + 16); one scale
                const int e0 = ch * 16, h = e0 >> 7, qq = (e0 & 127) >> 5, l0 = e0 & 31;
                const int sc = has_row ? (int)(int8_t)blk[192 + 8 * h + (l0 >> 4) + 2 * qq] : 0;
                int dg[3];
                q6_digits(sc, dg[0], dg[1], dg[2]);
                uint32_t w[3][4];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    uint32_t a[3] = {0, 0, 0};
#pragma unroll
                    for (int v = 0; v < 4; v++) {
                        const int l = l0 + 4 * u + v;
                        int q = 0;
                        if (has_row) {
                            const int lowb = (qq & 1) ? blk[64 * h + l + 32] : blk[64 * h + l];
                            const int low = (qq >> 1) ? (lowb >> 4) : (lowb & 15);
                            q = (low | (((blk[128 + 32 * h + l] >> (2 * qq)) & 3) << 4)) - 32;
                        }
#pragma unroll
                        for (int pl = 0; pl < 3; pl++) a[pl] |= (uint32_t)(q * dg[pl] & 0xFF) << (8 * v);
                    }
#pragma unroll
                    for (int pl = 0; pl < 3; pl++) w[pl][u] = a[pl];
                }
#pragma unroll
                for (int pl = 0; pl < 3; pl++)
                    *(uint4 *)(planes + pl * kPlaneBytes + canon(row, e0, TM)) =
                        make_uint4(w[pl][0], w[pl][1], w[pl][2], w[pl][3]);
            }
        }
        // ---- operands visible to the tensor cores; one thread issues the MMAs
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        fence_before_sync();
        __syncthreads();
        fence_after_sync();
        if (tid == 0) {
            for (int pl = 0; pl < P; pl++)
                for (int s = 0; s < 8; s++)  // K = 32 per instruction: chunks 2s, 2s + 1
                    mma_i8(tmem + (uint32_t)(pl * TN),
                           smem_desc(planes_s + pl * kPlaneBytes + (uint32_t)(2 * s * TM * 16), TM * 16, 128),
                           smem_desc(bt_s + (uint32_t)(2 * s * TN * 16), TN * 16, 128), s > 0 ? 1u : 0u);
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             smem_u32(bar))
                         : "memory");
        }
        failed = __syncthreads_or(!mbar_wait_bounded(bar, phase, p.status));
        if (failed) break;  // the commit never arrived: DEV_TIMEOUT is set
        phase ^= 1u;
        fence_after_sync();
        // ---- block sums back (lane = row) and the block-ordered chain
        {
            uint32_t acc[kPlanes][32];
            const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
            tmem_ld32(lane_base + 0, acc[0]);
            tmem_ld32(lane_base + TN, acc[1]);
            if (P == 3) tmem_ld32(lane_base + 2 * TN, acc[2]);
#pragma unroll
            for (int n = 0; n < TN; n++) {
                int S = (int)acc[0][n] + 8 * (int)acc[1][n];
                if (P == 3) S += 64 * (int)acc[2][n];
                const float dx = mdx[n];
                tot[n] = __fmaf_rn(__int2float_rn(S), __fmul_rn(d, dx), tot[n]);
                if (dt == Q4_K) {
                    int M = 0;
#pragma unroll
                    for (int j = 0; j < 8; j++) M += mn8[j] * (int)mxs[n * 8 + j];
                    off[n] = __fmaf_rn(__int2float_rn(M), __fmul_rn(dmin, dx), off[n]);
                }
                if (!mok[n]) tokbad |= 1u << n;
            }
        }
        fence_before_sync();
        __syncthreads();  // planes, B and TMEM free for the next block
    }

    // ---- outputs: tot - off (+ bias, + residual)
    const int grow = r0 + row;
    if (has_row && !failed && !rowbad) {
        const float bias = sg.bias ? sg.bias[grow] : 0.f;
        for (int n = 0; n < ntok; n++) {
            if (tokbad >> n & 1u) continue;
            float v = __fsub_rn(tot[n], off[n]);
            if (sg.bias) v = __fadd_rn(v, bias);
            if (sg.res) v = __fadd_rn(sg.res[(long long)(n0 + n) * sg.ldy + grow], v);
            sg.y[(long long)(n0 + n) * sg.ldy + grow] = v;
        }
    }
    // refused pairs: the GEMV's warp-collective f32 product, row by row
    const unsigned badr = __ballot_sync(0xFFFFFFFFu, has_row && rowbad);
    if (!failed && (badr || tokbad)) {
        for (int rr = 0; rr < 32; rr++) {
            const int gr = r0 + warp * 32 + rr;
            if (warp * 32 + rr >= nrow) break;
            for (int n = 0; n < ntok; n++) {
                if (!(badr >> rr & 1u) && !(tokbad >> n & 1u)) continue;
                float v = row_dot_f32(dt, sg.w + (long long)gr * rb, p.x + (long long)(n0 + n) * p.K, p.nb);
                if (sg.bias) v = __fadd_rn(v, sg.bias[gr]);
                if (sg.res) v = __fadd_rn(sg.res[(long long)(n0 + n) * sg.ldy + gr], v);
                if (lane == 0) sg.y[(long long)(n0 + n) * sg.ldy + gr] = v;
            }
        }
    }
    // after a timeout, give the MMAs in flight one more bounded wait before
    // the accumulator columns are released
    if (failed) mbar_wait_bounded(bar, phase, nullptr);
    fence_before_sync();
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

}  // namespace

bool gemm_a8_tc_ok(const GemvSeg *segs, int nseg, const ActQ8 &act, int rows, long long K) {
    if (rows < kTcMinRows || K <= 0 || K % 256 || nseg <= 0 || nseg > kMaxSegs) return false;
    if ((uintptr_t)act.q & 15) return false;  // 16-byte activation reads
    for (int i = 0; i < nseg; i++)
        if (segs[i].dt != Q4_K && segs[i].dt != Q6_K) return false;
    return true;
}

cudaError_t gemm_a8_tc_prepare() {
    static bool done = false;
    if (done) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(gemm_a8_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemTc);
    if (e == cudaSuccess) done = true;
    return e;
}

cudaError_t launch_gemm_a8_tc(const GemvSeg *segs, int nseg, const float *x, ActQ8 act, int rows, long long K,
                              unsigned *status, cudaStream_t st, bool pdl) {
    if (!gemm_a8_tc_ok(segs, nseg, act, rows, K)) return cudaErrorInvalidValue;
    TcParams p = {};
    p.nseg = nseg;
    int t = 0;
    for (int i = 0; i < nseg; i++) {
        p.seg[i] = segs[i];
        p.seg_t0[i] = t;
        t += (segs[i].n + TM - 1) / TM;
    }
    p.seg_t0[nseg] = t;
    if (t == 0) return cudaSuccess;
    p.act = act;
    p.x = x;
    p.rows = rows;
    p.K = K;
    p.nb = (int)(K / 256);
    p.status = status;
    cudaError_t e = gemm_a8_tc_prepare();
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[1];
    cfg.gridDim = dim3(t, (rows + TN - 1) / TN);
    cfg.blockDim = dim3(kThr);
    cfg.dynamicSmemBytes = kSmemTc;
    cfg.stream = st;
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemm_a8_tc_kernel, p);
}

}  // namespace mimgpu
