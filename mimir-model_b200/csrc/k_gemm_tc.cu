// k_gemm_tc.cu -- dequant_matmul_a8.v2 (block 256) for many activation rows
// (prompt processing, batched decode) on the 5th-generation tensor cores.
//
// Same results as the GEMV (k_gemv_a8.cu) and the reference's dotQ8KRef
// (internal/kernels/q8k_test.go:35-117 of gsoultan/mimir-model), bit for
// bit, as the reference's own prompt tile kernels are (amx.go:24-51,
// vnni.go:22-32): the exact int32 block sums S (and M for Q4_K), then the
// block-ordered f32 chain tot = fma(float(S), d*dx, tot),
// off = fma(float(M), dmin*dx, off), result tot - off.
//
// A CTA owns 128 weight rows (TMEM lanes) x NT activation rows (NT = 64, or
// 32 for launches of 16-32 rows).  For every 256-element block the rows'
// quants become int8 "digit planes" whose products with the int8
// activations are exact MMA operands, and tcgen05.mma kind::i8 (M 128,
// N NT, K 32) sums each plane over the block into TMEM:
//   Q4_K  sc = lo + 8 hi (3-bit digits): planes q*lo, q*hi in [0, 105] and
//         the sub-block mins m in [0, 63]:  S = P0 + 8 P1,  M = P2;
//   Q6_K  sc = d0 + 8 d1 + 64 d2 (digits in [-3, 4]): planes (q-32)*d in
//         [-128, 124]:  S = P0 + 8 P1 + 64 P2.
// Data flow per block: the tile's raw weight blocks and the block's
// activation tile arrive by TMA in a 4-slot input ring; warps 1-4 (one
// weight row per thread, the thread's TMEM lane) unpack their rows a
// quarter block at a time into the planes, written straight into TMEM with
// tcgen05.st (two plane stages of one quarter, or of half a block when
// NT = 32), so the MMA reads A from TMEM and only the activation tile from
// shared memory; once every decoder has filled a stage, the MMA thread
// (warp 0) issues its MMAs into one of two TMEM accumulator sets and
// commits them to the barriers that free the stage and hand the set on; it
// never waits on the tensor pipe itself.  Warps 5-12 (one row and NT/2
// activation rows per thread) read the sums back with tcgen05.ld, convert
// them exactly and continue the block-ordered chain in registers, and
// write the outputs at the end (bias, residual, refused pairs); one of them
// refills each input slot as soon as its block's MMAs are complete.
// Every wait is bounded (2 s, or sooner once another role has given up):
// the kernel then sets DEV_TIMEOUT, drains the MMAs it issued, frees TMEM
// and returns.
#include <cuda.h>  // CUtensorMap (types only)

#include <algorithm>
#include <cstdint>

#include "a8_refused.cuh"
#include "common.cuh"
#include "kernels.h"

namespace mimgpu {

void *tmap_encode_fn();  // cuTensorMapEncodeTiled from the driver (k_gemv_a8.cu)

namespace {

constexpr int TM = 128;                          // weight rows per CTA = MMA M = TMEM lanes
constexpr int kNTMax = 64;                       // activation rows per CTA = MMA N: 64, or 32 for 16-32 rows
constexpr int kPlanes = 3;
constexpr int kQuarter = 64;                     // K elements per plane stage
constexpr int kMaxStages = 4;                    // plane stages in TMEM (TcCfg::kStages)
constexpr int kNin = 4;                          // input ring slots
constexpr int kRawPitch = 240;                   // Q6_K box width: a 210-byte block from its 16-byte boundary
constexpr int kMeta = 4;                         // per-block scale ring between decoders and epilogue
constexpr int kDec = 128, kEpi = 256;
constexpr int kThreads = 32 + kDec + kEpi;
constexpr uint32_t kAStageCols = kPlanes * kQuarter / 4;  // 4 int8 per 32-bit column
constexpr uint32_t kTmemCols = 512;
constexpr int kOffMeta = 256;
constexpr int kOffIn = 7168;

// The shapes that depend on the activation tile NT.  With NT = 32 the two
// accumulator sets take 192 TMEM columns, which leaves room for plane
// stages of half a block.
template <int NT>
struct TcCfg {
    // kStages plane stages of kGroup quarters each: with NT = 32 a stage is
    // half a block, so the MMA thread waits and commits once per 12 MMAs
    static constexpr int kStages = 2;
    static constexpr int kGroup = NT == 32 ? 2 : 1;
    static constexpr int kBBlock = NT * 256;     // activation tile of one block: two 128-byte-swizzled boxes
    static constexpr int kInQ4 = TM * 144 + kBBlock;  // input slot: raw rows, then the activation tile
    static constexpr int kInQ6 = TM * kRawPitch + kBBlock;
    static constexpr int kEpiTok = NT / 2;       // activation rows per epilogue thread
    static constexpr uint32_t kAccCols = kPlanes * NT;  // one accumulator set
    static constexpr uint32_t kACol0 = 2 * kAccCols;    // plane stages after the two accumulator sets
    static constexpr int kSmem = kOffIn + kNin * kInQ6;
    // kind::i8 instruction descriptor: D s32, A and B signed 8-bit, K-major, N = NT, M = TM
    static constexpr uint32_t kIdesc =
        (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(NT >> 3) << 17) | ((uint32_t)(TM >> 4) << 24);
    static_assert(NT == 32 || NT == 64, "activation tile");
    static_assert(kStages <= kMaxStages, "plane stages");
    static_assert(kACol0 + kStages * kGroup * kAStageCols <= kTmemCols, "TMEM columns");
    static_assert(kOffIn % 1024 == 0 && kInQ4 % 1024 == 0 && kInQ6 % 1024 == 0, "alignment");
    static_assert(kSmem <= 227 * 1024, "shared memory");
};

struct Meta {
    float d[TM], dmin[TM];
    float dx[kNTMax];
    int ok[kNTMax];
};

struct Bars {
    uint64_t full[kMaxStages], empty[kMaxStages];
    uint64_t accfull[2], accempty[2];
    uint64_t infull[kNin], inempty[kNin];
    uint64_t metafull[kMeta], metaempty[kMeta];
    uint64_t drain;
    uint32_t tmem;
    int abort;
};

static_assert(sizeof(Bars) <= kOffMeta, "barrier block");
static_assert(kOffMeta + kMeta * (int)sizeof(Meta) <= kOffIn, "meta ring");

struct TcParams {
    CUtensorMap tmap[kMaxSegs];  // raw weights [n, row bytes] u8, box [box width, 128]
    CUtensorMap amap;            // activation quants [rows, K] u8, box [128, 64], 128-byte swizzle
    GemvSeg seg[kMaxSegs];
    int seg_t0[kMaxSegs + 1];    // first 128-row tile of each segment
    int nseg;
    ActQ8 act;
    const float *x;              // f32 activations (refused pairs)
    int rows;
    long long K;
    int nb;
    unsigned *status;
    // split launches (REC): each CTA's exact block sums (S, M) go to
    // rec[seg_rec0[s] + (kb * rows + t) * n_s + row] and the row's block
    // scales (d, dmin) to dd[seg_dd0[s] + kb * n_s + row], for the chain kernel
    int2 *rec;
    float2 *dd;
    long long seg_rec0[kMaxSegs], seg_dd0[kMaxSegs];
};

// byte offset of (row, 16-byte K chunk c) in a K-major no-swizzle operand of
// R rows: core matrices of 8 rows x 16 bytes, 8-row groups 128 bytes apart
// (SBO), K chunks R*16 bytes apart (LBO)
__device__ __forceinline__ uint32_t canon(int row, int c, int R) {
    return (uint32_t)((c * (R >> 3) + (row >> 3)) * 128 + (row & 7) * 16);
}

__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);  // version 1, no swizzle
}

// K-major operand in the 128-byte swizzle layout (what a TMA box of 128-byte
// rows with CU_TENSOR_MAP_SWIZZLE_128B writes): 8-row atoms of 1024 bytes
// (SBO), 1024-byte aligned; K steps inside an atom advance the start address
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}

// D (TMEM) += A (TMEM: lane = row, 4 int8 of K per column) x B (shared memory);
// kIdesc: the kind::i8 instruction descriptor (TcCfg)
template <uint32_t kIdesc>
__device__ __forceinline__ void mma_i8_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(kIdesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ uint4 ld16(const uint8_t *p) { return *(const uint4 *)p; }
__device__ __forceinline__ void st16(uint8_t *p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    *(uint4 *)p = make_uint4(a, b, c, d);
}

// Bounded wait that also gives up once another role has: false means the
// kernel is aborting (DEV_TIMEOUT is set by whoever timed out first).
__device__ __forceinline__ bool wait_bar(uint64_t *bar, uint32_t parity, Bars &B, unsigned *status) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns(), limit = dev_wait_limit(status);
    for (uint32_t i = 1;; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255) == 0) {
            if (*(volatile int *)&B.abort) return false;
            if (global_ns() - t0 > limit) {
                *(volatile int *)&B.abort = 1;
                atomicOr(status, (unsigned)DEV_TIMEOUT);
                return false;
            }
        }
    }
}

// exact int -> f32 for |v| < 2^22
__device__ __forceinline__ float small_i2f(uint32_t v) {
    return __fsub_rn(__int_as_float((int)(v + 0x4B400000u)), 12582912.0f);
}

// Digits of a Q6_K scale in base 8, each in [-3, 4]: sc = d0 + 8 d1 + 64 d2.
__device__ __forceinline__ void q6_digits(int sc, int (&dg)[3]) {
    dg[0] = ((sc + 3) & 7) - 3;
    const int t = (sc - dg[0]) >> 3;
    dg[1] = ((t + 3) & 7) - 3;
    dg[2] = (t - dg[1]) >> 3;
}

// ------------------------------------------------------------ decode: Q4_K
// The thread's row, quarter qi (elements 64qi..64qi+63: qs bytes
// [32qi, 32qi+32), low nibbles then high nibbles) of the block at `blk`
// (144 bytes, 16-byte aligned in shared memory), as the three planes' 16
// columns at TMEM address `ta` (this warp's lanes).
__device__ __forceinline__ void decode_q4k_quarter(const uint8_t *blk, int qi, uint32_t ta) {
    const uint4 hdr = ld16(blk);
    const uint32_t sw[3] = {hdr.y, hdr.z, hdr.w};
    const uint4 g0 = ld16(blk + 16 + 32 * qi), g1 = ld16(blk + 32 + 32 * qi);
    const uint32_t qw[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
    uint32_t a0[16], a1[16], mp[16];
#pragma unroll
    for (int up = 0; up < 2; up++) {  // sub-block 2qi + up
        int sc, m;
        q4k_scale_min(sw, 2 * qi + up, sc, m);
        const uint32_t lo = (uint32_t)(sc & 7), hi = (uint32_t)(sc >> 3), mw = (uint32_t)m * 0x01010101u;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const uint32_t nib = up ? ((qw[k] >> 4) & 0x0F0F0F0Fu) : (qw[k] & 0x0F0F0F0Fu);
            a0[8 * up + k] = nib * lo;  // bytes q*lo <= 105: no carries
            a1[8 * up + k] = nib * hi;
            mp[8 * up + k] = mw;
        }
    }
    tmem_st16(ta, a0);
    tmem_st16(ta + kQuarter / 4, a1);
    tmem_st16(ta + 2 * kQuarter / 4, mp);
}

// ------------------------------------------------------------ decode: Q6_K
// The block starts at byte 4*WO + sh/8 of the 16-byte aligned window `win`
// (sh is 0 or 16: blocks are 2-byte aligned).  Quarter qi is half h = qi/2,
// quarters qq = 2(qi&1), 2(qi&1)+1 of it: scales 8h + 4(qi&1) .. +4.
template <int WO>
__device__ __forceinline__ void decode_q6k_quarter(const uint8_t *win, int sh, int qi, uint32_t ta) {
    const int h = qi >> 1, odd = qi & 1;
    // ql bytes [64h, 64h+64): window chunks 4h..4h+4
    uint32_t u[20];
#pragma unroll
    for (int i = 0; i < 5; i++) {
        const uint4 v = ld16(win + 64 * h + 16 * i);
        u[4 * i] = v.x; u[4 * i + 1] = v.y; u[4 * i + 2] = v.z; u[4 * i + 3] = v.w;
    }
    uint32_t ql[16];
#pragma unroll
    for (int i = 0; i < 16; i++) ql[i] = __funnelshift_r(u[WO + i], u[WO + i + 1], sh);
    // qh bytes [128 + 32h, +32): window chunks 8+2h..10+2h
    uint32_t v3[12];
#pragma unroll
    for (int i = 0; i < 3; i++) {
        const uint4 v = ld16(win + 128 + 32 * h + 16 * i);
        v3[4 * i] = v.x; v3[4 * i + 1] = v.y; v3[4 * i + 2] = v.z; v3[4 * i + 3] = v.w;
    }
    uint32_t qh[8];
#pragma unroll
    for (int i = 0; i < 8; i++) qh[i] = __funnelshift_r(v3[WO + i], v3[WO + i + 1], sh);
    // the quarter's 4 scales: bytes [192 + 8h + 4 odd, +4): window chunks 12, 13
    const uint4 s0 = ld16(win + 192), s1 = ld16(win + 208);
    const uint32_t t[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    const int wi = 2 * h + odd;  // word of the scales relative to the block's scale region
    const uint32_t scw = __funnelshift_r(wi == 0 ? t[WO] : wi == 1 ? t[WO + 1] : wi == 2 ? t[WO + 2] : t[WO + 3],
                                         wi == 0 ? t[WO + 1] : wi == 1 ? t[WO + 2] : wi == 2 ? t[WO + 3] : t[WO + 4], sh);
    uint32_t w[3][16];
#pragma unroll
    for (int cc = 0; cc < 4; cc++) {
        // elements 64qi + 16cc ..: quarter qq = 2 odd + cc/2, l in [16(cc&1), +16), scale byte cc
        const int qq = 2 * odd + (cc >> 1), g = 2 * (qq & 1) + (cc & 1);
        const int sc = (int)(int8_t)((scw >> (8 * cc)) & 0xFF);
        int dg[3];
        q6_digits(sc, dg);
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const uint32_t q = ((ql[4 * g + k] >> (4 * (qq >> 1))) & 0x0F0F0F0Fu) |
                               (((qh[4 * (cc & 1) + k] >> (2 * qq)) & 0x03030303u) << 4);
            const uint32_t xa = __byte_perm(q, 0, 0x4140), xb = __byte_perm(q, 0, 0x4342);  // 16-bit lanes
#pragma unroll
            for (int p = 0; p < 3; p++) {
                // lanes (q-32)*d + 256 in [128, 380]: their low bytes are the int8 products
                const uint32_t c = (uint32_t)(256 - 32 * dg[p]) * 0x00010001u;
                const uint32_t ra = xa * (uint32_t)dg[p] + c, rb = xb * (uint32_t)dg[p] + c;
                w[p][4 * cc + k] = __byte_perm(ra, rb, 0x6420);
            }
        }
    }
    tmem_st16(ta, w[0]);
    tmem_st16(ta + kQuarter / 4, w[1]);
    tmem_st16(ta + 2 * kQuarter / 4, w[2]);
}

// One block of the chain for the thread's row and its NT/2 activation rows:
// the block sums from TMEM (accumulator columns from `col`, this warp's
// lanes), converted exactly and folded in block order.
template <int NT, bool Q4, int kEpiTok = TcCfg<NT>::kEpiTok>
__device__ __forceinline__ void epi_block(uint32_t col, const float *dxs, float d, float dmin,
                                          float (&tot)[kEpiTok], float (&off)[kEpiTok]) {
#pragma unroll
    for (int c = 0; c < kEpiTok / 16; c++) {
        float dx[16];
#pragma unroll
        for (int j4 = 0; j4 < 4; j4++) {
            const float4 v = *(const float4 *)(dxs + 16 * c + 4 * j4);
            dx[4 * j4] = v.x; dx[4 * j4 + 1] = v.y; dx[4 * j4 + 2] = v.z; dx[4 * j4 + 3] = v.w;
        }
        uint32_t a0[16], a1[16];
        tmem_ld16(col + 16 * c, a0);
        tmem_ld16(col + NT + 16 * c, a1);
        tmem_wait_ld();
        if (Q4) {
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const float fs = __fmaf_rn(small_i2f(a1[j]), 8.0f, small_i2f(a0[j]));  // = float(P0 + 8 P1)
                tot[16 * c + j] = __fmaf_rn(fs, __fmul_rn(d, dx[j]), tot[16 * c + j]);
            }
            tmem_ld16(col + 2 * NT + 16 * c, a0);  // the mins plane
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; j++)
                off[16 * c + j] = __fmaf_rn(small_i2f(a0[j]), __fmul_rn(dmin, dx[j]), off[16 * c + j]);
        } else {
#pragma unroll
            for (int j = 0; j < 16; j++) a0[j] += 8u * a1[j];
            tmem_ld16(col + 2 * NT + 16 * c, a1);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const int S = (int)(a0[j] + 64u * a1[j]);
                tot[16 * c + j] = __fmaf_rn(__int2float_rn(S), __fmul_rn(d, dx[j]), tot[16 * c + j]);
            }
        }
    }
}

__device__ __forceinline__ void tma_2d(const CUtensorMap *map, uint8_t *dst, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"((const void *)map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// REC: a split launch (gridDim.z parts of the K axis): the epilogue stores
// each block's exact sums to p.rec instead of folding them; the chain
// kernel then runs the block-ordered fused multiply-adds.
template <int NT, bool REC>
__global__ void __launch_bounds__(kThreads, 1) gemm_a8_tc_kernel(const __grid_constant__ TcParams p) {
    using Cf = TcCfg<NT>;
    constexpr int kStages = Cf::kStages, kGroup = Cf::kGroup, kBBlock = Cf::kBBlock, kInQ4 = Cf::kInQ4,
                  kInQ6 = Cf::kInQ6;
    constexpr int kGroups = 4 / kGroup;  // plane stages per block
    constexpr int kEpiTok = Cf::kEpiTok;
    constexpr uint32_t kAccCols = Cf::kAccCols, kACol0 = Cf::kACol0;
    extern __shared__ __align__(1024) uint8_t sm[];
    Bars &B = *(Bars *)sm;
    Meta *meta = (Meta *)(sm + kOffMeta);
    uint8_t *inring = sm + kOffIn;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    // the tile: segment, its 128 rows, the NT activation rows
    const int tile = blockIdx.y;
    int si = 0;
    while (si + 1 < p.nseg && tile >= p.seg_t0[si + 1]) si++;
    GemvSeg sg = p.seg[0];
    const CUtensorMap *map = &p.tmap[0];
#pragma unroll
    for (int i = 1; i < kMaxSegs; i++)
        if (i == si) {
            sg = p.seg[i];
            map = &p.tmap[i];
        }
    const int r0 = (tile - p.seg_t0[si]) * TM, nrow = min(TM, sg.n - r0);
    const int n0 = blockIdx.x * NT, ntok = min(NT, p.rows - n0);
    const int dt = sg.dt, bb = block_bytes(dt);
    // this CTA's blocks [kb0, kb0 + nb) of the K axis: all of them, or its
    // part of a split launch (REC); loops run over the local index kb
    const int kb0 = REC ? (int)((long long)p.nb * blockIdx.z / gridDim.z) : 0;
    const int nb = REC ? (int)((long long)p.nb * (blockIdx.z + 1) / gridDim.z) - kb0 : p.nb;
    const bool q4 = dt == Q4_K;
    const int pitch = q4 ? 144 : kRawPitch;      // raw box width = row pitch in the slot
    const int nin = kNin;
    const int inbytes = q4 ? kInQ4 : kInQ6;
    const uint32_t rawbox = (uint32_t)(pitch * TM);

    if (tid == 0) {
        for (int i = 0; i < kStages; i++) {
            mbar_init(&B.full[i], kDec);
            mbar_init(&B.empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&B.accfull[i], 1);
            mbar_init(&B.accempty[i], kEpi);
        }
        for (int i = 0; i < kNin; i++) {
            mbar_init(&B.infull[i], 1);
            mbar_init(&B.inempty[i], kDec);  // the decoders are done with the raw rows
        }
        for (int i = 0; i < kMeta; i++) {
            mbar_init(&B.metafull[i], kDec);
            mbar_init(&B.metaempty[i], kEpi);
        }
        mbar_init(&B.drain, 1);
        B.abort = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&B.tmem)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = B.tmem;
    pdl_launch_dependents();

    // block kb's inputs into slot kb % nin: raw weights, then the activation tile
    auto fetch_raw = [&](int kb) {
        uint8_t *slot = inring + (kb % nin) * inbytes;
        mbar_arrive_expect_tx(&B.infull[kb % nin], rawbox + (uint32_t)kBBlock);
        tma_2d(map, slot, ((kb0 + kb) * bb) & ~15, r0, &B.infull[kb % nin]);
    };
    auto fetch_act = [&](int kb) {  // two boxes of NT rows x 128 bytes
        uint8_t *slot = inring + (kb % nin) * inbytes + TM * pitch;
        tma_2d(&p.amap, slot, (kb0 + kb) * 256, n0, &B.infull[kb % nin]);
        tma_2d(&p.amap, slot + NT * 128, (kb0 + kb) * 256 + 128, n0, &B.infull[kb % nin]);
    };
    if (warp == 0) {
        // ------------------------------------------------------- MMA issue
        // (the input slots are refilled by the epilogue, which sees each
        // block's MMAs complete: this thread never waits on the tensor pipe)
        if (lane == 0) {
            for (int kb = 0; kb < min(nin, nb); kb++) fetch_raw(kb);  // weights are read-only
            pdl_wait();
            for (int kb = 0; kb < min(nin, nb); kb++) fetch_act(kb);
            const uint32_t in0 = smem_u32(inring) + (uint32_t)(TM * pitch);
            bool ok = true;
            for (int kb = 0; kb < nb && ok; kb++) {
                const int j = kb % nin, b = kb & 1;
                if (!wait_bar(&B.accempty[b], ((kb >> 1) & 1) ^ 1, B, p.status)) break;
                const uint32_t dcol = tmem + (uint32_t)(b * kAccCols);
                for (int g = 0; g < kGroups; g++) {
                    const int i = kGroups * kb + g, s = i % kStages;
                    if (!wait_bar(&B.full[s], (i / kStages) & 1, B, p.status)) {
                        ok = false;
                        break;
                    }
                    fence_after_sync();
#pragma unroll
                    for (int u = 0; u < kGroup; u++) {
                        const int qi = g * kGroup + u;
                        // quarter qi: box qi/2, bytes 64 (qi&1) + 32 ks of each 128-byte row
                        const uint64_t bd =
                            smem_desc_sw128(in0 + (uint32_t)(j * inbytes + (qi >> 1) * NT * 128 + (qi & 1) * 64));
                        const uint32_t acol = tmem + kACol0 + (uint32_t)((s * kGroup + u) * kAStageCols);
#pragma unroll
                        for (int pl = 0; pl < kPlanes; pl++) {
                            mma_i8_ts<Cf::kIdesc>(dcol + pl * NT, acol + pl * (kQuarter / 4), bd, qi ? 1u : 0u);
                            mma_i8_ts<Cf::kIdesc>(dcol + pl * NT, acol + pl * (kQuarter / 4) + 8, bd + 2,
                                                  1u);  // + 32 bytes
                        }
                    }
                    mma_commit(&B.empty[s]);
                }
                if (ok) mma_commit(&B.accfull[b]);
            }
            // every MMA issued has completed before TMEM is released
            mma_commit(&B.drain);
            mbar_wait_bounded(&B.drain, 0, p.status);
        }
        __syncwarp();
    } else if (warp <= 4) {
        // ------------------------------------------------------- decoders
        const int r = 32 * (warp & 3) + lane;  // row = TMEM lane (warp w reaches lanes 32(w%4)..)
        const uint32_t ta0 = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + kACol0;
        pdl_wait();
        // activation-row scales, one block ahead
        float dx_next = 0.f;
        int ok_next = 1;
        if (r < ntok) {
            dx_next = p.act.dx[(long long)(n0 + r) * p.nb + kb0];
            ok_next = p.act.ok[(long long)(n0 + r) * p.nb + kb0];
        }
        for (int kb = 0; kb < nb; kb++) {
            const int j = kb % nin, ms = kb % kMeta;
            // tcgen05.st is warp-collective: the warp goes on only if every lane's waits succeeded
            const bool got = wait_bar(&B.infull[j], (kb / nin) & 1, B, p.status) &&
                             wait_bar(&B.metaempty[ms], ((kb / kMeta) & 1) ^ 1, B, p.status);
            if (!__all_sync(0xFFFFFFFFu, got)) break;
            const int ph = ((kb0 + kb) * bb) & 15;
            const uint8_t *win = inring + j * inbytes + r * pitch;
            // per-block scales of the row and of the activation rows
            Meta &m = meta[ms];
            if (q4) {
                const uint32_t dm = *(const uint32_t *)win;
                m.d[r] = f16_to_f32(dm & 0xFFFFu);
                m.dmin[r] = f16_to_f32(dm >> 16);
            } else {
                const uint32_t wd = *(const uint32_t *)(win + ((ph + 208) & ~3));
                m.d[r] = f16_to_f32((wd >> (8 * (ph & 3))) & 0xFFFFu);
                m.dmin[r] = 0.f;
            }
            if (r < NT) {
                m.dx[r] = dx_next;
                m.ok[r] = ok_next;
                if (r < ntok && kb + 1 < nb) {
                    dx_next = p.act.dx[(long long)(n0 + r) * p.nb + kb0 + kb + 1];
                    ok_next = p.act.ok[(long long)(n0 + r) * p.nb + kb0 + kb + 1];
                }
            }
            mbar_arrive(&B.metafull[ms]);
            bool ok = true;
            for (int qi = 0; qi < 4; qi++) {
                const int i = kGroups * kb + qi / kGroup, s = i % kStages, u = qi % kGroup;
                if (u == 0 &&
                    !__all_sync(0xFFFFFFFFu, wait_bar(&B.empty[s], ((i / kStages) & 1) ^ 1, B, p.status))) {
                    ok = false;
                    break;
                }
                if (u == 0) fence_after_sync();
                const uint32_t ta = ta0 + (uint32_t)((s * kGroup + u) * kAStageCols);
                if (q4) {
                    decode_q4k_quarter(win, qi, ta);
                } else {
                    const int sh = 8 * (ph & 3);
                    switch (ph >> 2) {
                    case 0: decode_q6k_quarter<0>(win, sh, qi, ta); break;
                    case 1: decode_q6k_quarter<1>(win, sh, qi, ta); break;
                    case 2: decode_q6k_quarter<2>(win, sh, qi, ta); break;
                    default: decode_q6k_quarter<3>(win, sh, qi, ta); break;
                    }
                }
                if (u == kGroup - 1) {  // the stage is written: its MMAs may go
                    tmem_wait_st();
                    fence_before_sync();
                    mbar_arrive(&B.full[s]);
                }
            }
            if (!ok) break;
            mbar_arrive(&B.inempty[j]);  // this thread is done with the slot's raw rows
        }
    } else {
        // ------------------------------------------------------- epilogue
        const int q = warp & 3;                  // TMEM lane quarter (warp % 4): rows 32q..32q+31
        const int th = (warp - 5) >> 2;          // activation rows 32th..32th+31
        const int r = 32 * q + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(th * kEpiTok);
        pdl_wait();
        float tot[kEpiTok], off[kEpiTok];
#pragma unroll
        for (int n = 0; n < kEpiTok; n++) tot[n] = off[n] = 0.f;
        bool rowbad = false, done = true;
        uint32_t tokbad = 0;
        for (int kb = 0; kb < nb; kb++) {
            const int b = kb & 1, ms = kb % kMeta;
            // tcgen05.ld is warp-collective: the warp goes on only if every lane's waits succeeded
            const bool got = wait_bar(&B.metafull[ms], (kb / kMeta) & 1, B, p.status) &&
                             wait_bar(&B.accfull[b], (kb >> 1) & 1, B, p.status);
            if (!__all_sync(0xFFFFFFFFu, got)) {
                done = false;
                break;
            }
            fence_after_sync();
            if (warp == 5 && kb + nin < nb) {
                // block kb's MMAs are complete, so its slot's activation tile is
                // free; once the decoders are done with its raw rows (long
                // before), the slot takes block kb + nin
                if (lane == 0 && wait_bar(&B.inempty[kb % nin], (kb / nin) & 1, B, p.status)) {
                    fetch_raw(kb + nin);
                    fetch_act(kb + nin);
                }
                __syncwarp();
            }
            if (REC) {
                // the block's exact sums of the row and its NT/2 activation rows
                static_assert(!REC || kEpiTok == 16, "records from one 16-column load per plane");
                const uint32_t col = lane_base + (uint32_t)(b * kAccCols);
                uint32_t a0[16], a1[16], a2[16];
                tmem_ld16(col, a0);
                tmem_ld16(col + NT, a1);
                tmem_ld16(col + 2 * NT, a2);
                tmem_wait_ld();
                fence_before_sync();
                mbar_arrive(&B.accempty[b]);
                if (r < nrow) {
                    if (th == 0) {
                        const Meta &m = meta[ms];
                        p.dd[p.seg_dd0[si] + (long long)(kb0 + kb) * sg.n + r0 + r] = make_float2(m.d[r], m.dmin[r]);
                    }
                    int2 *rc = p.rec + p.seg_rec0[si] + ((long long)(kb0 + kb) * p.rows + n0 + th * kEpiTok) * sg.n + r0 + r;
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        if (th * kEpiTok + j >= ntok) break;
                        const int S = q4 ? (int)(a0[j] + 8u * a1[j]) : (int)(a0[j] + 8u * a1[j] + 64u * a2[j]);
                        rc[(long long)j * sg.n] = make_int2(S, q4 ? (int)a2[j] : 0);
                    }
                }
                mbar_arrive(&B.metaempty[ms]);
                continue;
            }
            const Meta &m = meta[ms];
            const float d = m.d[r], dmin = m.dmin[r];
            rowbad |= !isfinite(d) || !isfinite(dmin);
            const uint32_t col = lane_base + (uint32_t)(b * kAccCols);
            if (dt == Q4_K)
                epi_block<NT, true>(col, m.dx + th * kEpiTok, d, dmin, tot, off);
            else
                epi_block<NT, false>(col, m.dx + th * kEpiTok, d, dmin, tot, off);
            fence_before_sync();
            mbar_arrive(&B.accempty[b]);
#pragma unroll
            for (int n = 0; n < kEpiTok; n++)
                if (!m.ok[th * kEpiTok + n]) tokbad |= 1u << n;
            mbar_arrive(&B.metaempty[ms]);
        }
        if (!REC && __all_sync(0xFFFFFFFFu, done)) {
            // outputs: tot - off (+ bias, + residual) ...
            const int grow = r0 + r, t0 = n0 + th * kEpiTok, nt = min(kEpiTok, ntok - th * kEpiTok);
            if (r < nrow && !rowbad) {
                const float bias = sg.bias ? sg.bias[grow] : 0.f;
#pragma unroll
                for (int n = 0; n < kEpiTok; n++) {
                    if (n >= nt) break;
                    if (tokbad >> n & 1u) continue;
                    float v = __fsub_rn(tot[n], off[n]);
                    if (sg.bias) v = __fadd_rn(v, bias);
                    if (sg.res) v = __fadd_rn(sg.res[(long long)(t0 + n) * sg.ldy + grow], v);
                    sg.y[(long long)(t0 + n) * sg.ldy + grow] = v;
                }
            }
            // ... and the refused pairs: the GEMV's warp-collective f32 product
            const unsigned badr = __ballot_sync(0xFFFFFFFFu, r < nrow && rowbad);
            if (badr || tokbad) {
                for (int rr = 0; rr < 32 && 32 * q + rr < nrow; rr++) {
                    const int gr = r0 + 32 * q + rr;
                    for (int n = 0; n < nt; n++) {
                        if (!(badr >> rr & 1u) && !(tokbad >> n & 1u)) continue;
                        float v = row_dot_f32(dt, sg.w + (long long)gr * row_bytes(dt, p.K),
                                              p.x + (long long)(t0 + n) * p.K, p.nb);
                        if (sg.bias) v = __fadd_rn(v, sg.bias[gr]);
                        if (sg.res) v = __fadd_rn(sg.res[(long long)(t0 + n) * sg.ldy + gr], v);
                        if (lane == 0) sg.y[(long long)(t0 + n) * sg.ldy + gr] = v;
                    }
                }
            }
        }
    }
    fence_before_sync();
    __syncthreads();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// [n, row bytes] u8 map of a weight matrix, box [one block from its 16-byte
// boundary, 128 rows], zero fill past either edge
bool raw_tmap(const GemvSeg &sg, long long K, CUtensorMap *out) {
    const EncodeTiledFn fn = (EncodeTiledFn)tmap_encode_fn();
    if (!fn) return false;
    const long long rb = row_bytes(sg.dt, K);
    const cuuint64_t dims[2] = {(cuuint64_t)rb, (cuuint64_t)sg.n};
    const cuuint64_t strides[1] = {(cuuint64_t)rb};
    const cuuint32_t boxd[2] = {(cuuint32_t)(sg.dt == Q4_K ? 144 : kRawPitch), (cuuint32_t)TM};
    const cuuint32_t estr[2] = {1, 1};
    return fn(out, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void *)sg.w, dims, strides, boxd, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [rows, K] u8 map of the activation quants, box [128 bytes, NT rows] in the
// 128-byte swizzle: one box is the MMA's B operand for half a block
bool act_tmap(const int8_t *q, int rows, long long K, int NT, CUtensorMap *out) {
    const EncodeTiledFn fn = (EncodeTiledFn)tmap_encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K};
    const cuuint32_t boxd[2] = {128, (cuuint32_t)NT};
    const cuuint32_t estr[2] = {1, 1};
    return fn(out, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void *)q, dims, strides, boxd, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The second half of a split launch: for every (weight row, activation
// row) pair, the block-ordered chain of dotQ8KRef over the records of the
// split CTAs -- tot = fma(float(S), d*dx, tot), off = fma(float(M),
// dmin*dx, off) -- then bias and residual, exactly as the unsplit
// epilogue; pairs either side refuses take the f32 product.  A CTA is 32
// consecutive weight rows (the lanes) x 8 activation rows (the warps).
struct ChainParams {
    GemvSeg seg[kMaxSegs];
    int seg_n0[kMaxSegs + 1];      // first row of each segment in the launch's row order
    long long seg_rec0[kMaxSegs];  // its records in rec
    long long seg_dd0[kMaxSegs];   // its block scales in dd
    int nseg;
    const int2 *rec;
    const float2 *dd;
    ActQ8 act;
    const float *x;
    int rows;
    long long K;
    int nb;
};

__global__ void __launch_bounds__(256) gemm_a8_chain_kernel(const __grid_constant__ ChainParams p) {
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.y * 8 + (threadIdx.x >> 5);  // warp-uniform
    const int gn = blockIdx.x * 32 + lane;
    const int total = p.seg_n0[p.nseg];
    auto seg_of = [&](int g) {
        int si = 0;
        while (si + 1 < p.nseg && g >= p.seg_n0[si + 1]) si++;
        return si;
    };
    const bool valid = gn < total && t < p.rows;
    const int si = valid ? seg_of(gn) : 0;
    const GemvSeg &sg = p.seg[si];
    const int n = gn - p.seg_n0[si];
    float tot = 0.f, off = 0.f;
    bool bad = false;
    if (valid) {
        const bool q4 = sg.dt == Q4_K;
        const int2 *rc = p.rec + p.seg_rec0[si] + (long long)t * sg.n + n;
        const float2 *ddp = p.dd + p.seg_dd0[si] + n;
        const long long kstride = (long long)p.rows * sg.n;
        const float *dxs = p.act.dx + (long long)t * p.nb;
        const int *oks = p.act.ok + (long long)t * p.nb;
#pragma unroll 8
        for (int kb = 0; kb < p.nb; kb++) {
            const int2 v = __ldcg(rc + kb * kstride);
            const float2 sc = __ldcg(ddp + (long long)kb * sg.n);
            const float dx = dxs[kb];
            const float d = sc.x, dmin = sc.y;
            bad |= !isfinite(d) || !isfinite(dmin) || !oks[kb];
            tot = __fmaf_rn(__int2float_rn(v.x), __fmul_rn(d, dx), tot);
            if (q4) off = __fmaf_rn(__int2float_rn(v.y), __fmul_rn(dmin, dx), off);
        }
        if (!bad) {
            float r = __fsub_rn(tot, off);
            if (sg.bias) r = __fadd_rn(r, sg.bias[n]);
            if (sg.res) r = __fadd_rn(sg.res[(long long)t * sg.ldy + n], r);
            sg.y[(long long)t * sg.ldy + n] = r;
        }
    }
    // refused pairs: the warp-collective f32 product of the GEMV and the GEMM
    unsigned rm = __ballot_sync(0xFFFFFFFFu, valid && bad);
    while (rm) {
        const int i = __ffs(rm) - 1;
        rm &= rm - 1;
        const int gi = blockIdx.x * 32 + i, sj = seg_of(gi);
        const GemvSeg &sgi = p.seg[sj];
        const int ni = gi - p.seg_n0[sj];
        float r = row_dot_f32(sgi.dt, sgi.w + (long long)ni * row_bytes(sgi.dt, p.K), p.x + (long long)t * p.K, p.nb);
        if (sgi.bias) r = __fadd_rn(r, sgi.bias[ni]);
        if (sgi.res) r = __fadd_rn(sgi.res[(long long)t * sgi.ldy + ni], r);
        if (lane == 0) sgi.y[(long long)t * sgi.ldy + ni] = r;
    }
}

// The K split of a launch of `tiles` row tiles and nb blocks: parts of at
// least 4 blocks that fill the SMs, when one part per tile leaves more
// than half of them idle; 1 = no split.
int split_parts(int tiles, int nb) {
    const int sms = num_sms();
    if (tiles <= 0 || 2 * tiles > sms) return 1;
    return std::max(1, std::min({sms / tiles, nb / 4, 8}));
}

}  // namespace

size_t gemm_a8_split_bytes(const GemvSeg *segs, int nseg, int rows, long long K) {
    if (rows < kTcMinRows || rows > 32 || K <= 0 || K % 256 || nseg <= 0 || nseg > kMaxSegs) return 0;
    int tiles = 0;
    long long n = 0;
    for (int i = 0; i < nseg; i++) {
        tiles += (segs[i].n + TM - 1) / TM;
        n += segs[i].n;
    }
    if (split_parts(tiles, (int)(K / 256)) < 2) return 0;
    // records, then the block scales
    return (size_t)n * (size_t)(K / 256) * ((size_t)rows * sizeof(int2) + sizeof(float2));
}

bool gemm_a8_tc_ok(const GemvSeg *segs, int nseg, const ActQ8 &act, int rows, long long K) {
    if (rows < kTcMinRows || K <= 0 || K % 256 || nseg <= 0 || nseg > kMaxSegs) return false;
    if ((uintptr_t)act.q & 15) return false;  // 2-D TMA of the activation quants
    for (int i = 0; i < nseg; i++) {
        if (segs[i].dt != Q4_K && segs[i].dt != Q6_K) return false;
        // 2-D TMA of the raw blocks: 16-byte aligned rows
        if (((uintptr_t)segs[i].w & 15) || row_bytes(segs[i].dt, K) % 16) return false;
    }
    return true;
}

cudaError_t gemm_a8_tc_prepare() {
    static std::atomic<unsigned long long> done{0};
    return once_per_device(done, [] {
        cudaError_t e = cudaFuncSetAttribute(gemm_a8_tc_kernel<64, false>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<64>::kSmem);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(gemm_a8_tc_kernel<32, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     TcCfg<32>::kSmem);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(gemm_a8_tc_kernel<32, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     TcCfg<32>::kSmem);
        return e;
    });
}

cudaError_t launch_gemm_a8_tc(const GemvSeg *segs, int nseg, const float *x, ActQ8 act, int rows, long long K,
                              unsigned *status, cudaStream_t st, bool pdl, const GemmSplit *split) {
    if (!gemm_a8_tc_ok(segs, nseg, act, rows, K)) return cudaErrorInvalidValue;
    TcParams p = {};
    p.nseg = nseg;
    int t = 0;
    for (int i = 0; i < nseg; i++) {
        p.seg[i] = segs[i];
        p.seg_t0[i] = t;
        t += (segs[i].n + TM - 1) / TM;
        if (segs[i].n > 0 && !raw_tmap(segs[i], K, &p.tmap[i])) return cudaErrorInvalidValue;
    }
    p.seg_t0[nseg] = t;
    if (t == 0) return cudaSuccess;
    // 16-32 activation rows: one tile of 32 (half the MMA work of 64, and
    // deeper plane staging); more: tiles of 64
    const int NT = rows <= 32 ? 32 : 64;
    if (!act_tmap(act.q, rows, K, NT, &p.amap)) return cudaErrorInvalidValue;
    p.act = act;
    p.x = x;
    p.rows = rows;
    p.K = K;
    p.nb = (int)(K / 256);
    p.status = status;
    cudaError_t e = gemm_a8_tc_prepare();
    if (e != cudaSuccess) return e;
    // few row tiles: split K over more CTAs when the caller gave room for
    // their records (records of n x rows x nb block sums)
    const size_t need = gemm_a8_split_bytes(segs, nseg, rows, K);
    const int parts = (need && split && split->rec && split->bytes >= need) ? split_parts(t, p.nb) : 1;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[1];
    cfg.gridDim = dim3((rows + NT - 1) / NT, t, parts);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = NT == 32 ? TcCfg<32>::kSmem : TcCfg<64>::kSmem;
    cfg.stream = st;
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    if (parts < 2)
        return NT == 32 ? cudaLaunchKernelEx(&cfg, gemm_a8_tc_kernel<32, false>, p)
                        : cudaLaunchKernelEx(&cfg, gemm_a8_tc_kernel<64, false>, p);
    ChainParams c = {};
    long long r0 = 0;
    int n0 = 0;
    for (int i = 0; i < nseg; i++) {
        p.seg_rec0[i] = c.seg_rec0[i] = r0;
        r0 += (long long)segs[i].n * rows * p.nb;
        c.seg[i] = segs[i];
        c.seg_n0[i] = n0;
        n0 += segs[i].n;
    }
    c.seg_n0[nseg] = n0;
    long long d0 = 0;
    for (int i = 0; i < nseg; i++) {
        p.seg_dd0[i] = c.seg_dd0[i] = d0;
        d0 += (long long)segs[i].n * p.nb;
    }
    c.nseg = nseg;
    p.rec = split->rec;
    c.rec = split->rec;
    // the scales after the records (8-byte aligned: records are 8 bytes each)
    p.dd = (float2 *)(split->rec + r0);
    c.dd = p.dd;
    c.act = act;
    c.x = x;
    c.rows = rows;
    c.K = K;
    c.nb = p.nb;
    cudaError_t e2 = cudaLaunchKernelEx(&cfg, gemm_a8_tc_kernel<32, true>, p);
    if (e2 != cudaSuccess) return e2;
    cudaLaunchConfig_t cc = {};
    cudaLaunchAttribute ca[1];
    cc.gridDim = dim3((n0 + 31) / 32, (rows + 7) / 8);
    cc.blockDim = dim3(256);
    cc.stream = st;
    ca[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    ca[0].val.programmaticStreamSerializationAllowed = 1;
    cc.attrs = ca;
    cc.numAttrs = 1;  // the records come from the launch just before, which it waits for
    return cudaLaunchKernelEx(&cc, gemm_a8_chain_kernel, c);
}

}  // namespace mimgpu
