// k_gemv_row.cu -- dequant_matmul_a8.v2 (block 256) for ONE activation row on
// sm_100a: the GEMV of a decode step.
//
// The same bits as gemv_a8_kernel (k_gemv_a8.cu) and dotQ8KRef
// (internal/kernels/q8k_test.go:35-117 of gsoultan/mimir-model): per 256-element
// block the exact int32 S = sum_s sc_s * sum(q*y) and (Q4_K) M = sum_s m_s * xs_s,
// then per row, in block order, tot = fma(float(S), d*dx, tot) and
// off = fma(float(M), dmin*dx, off); the result is tot - off, plus the bias,
// plus the residual.  Rows the reference refuses (linearA8,
// interp/fast.go:282-379) take the f32 product of a8_refused.cuh.
//
// Work decomposition: one CTA per SM: a producer thread, 16 consumer warps
// and two chain warps.
//  * Every matrix of the launch is cut into gridDim.x slabs of consecutive
//    rows, one per CTA, so each SM streams the same number of bytes (within
//    one row).  Rows are 16-byte multiples, so a slab is one contiguous byte
//    range; the producer streams it in stages of whole rows (the largest
//    multiple of the row's block count up to 256 blocks), one cp.async.bulk
//    per stage, into a ring of 3 to 8 data slots.  It starts before the
//    previous kernel has finished (weights are read-only), and refills a
//    slot as soon as the consumers have read it.
//  * The half-blocks of a stage go one to each consumer lane: Q4_K warps take
//    16 consecutive blocks, Q6_K warps the blocks 8i + (warp % 8) so that a
//    warp's 210-byte blocks share their 16-byte phase.  A stage holds whole
//    rows, so a lane meets the same block column in every stage.  The two
//    lanes of a block add their exact sums with one shuffle; the even lane
//    stores the block's (float(S), d*dx, float(M), dmin*dx) in a ring of
//    per-row records with its own stages, separate from the data slots.
//  * Chain warp c takes the record stages c, c + 2, ...: the block-ordered
//    chain over each row's records (one row per lane), bias, residual,
//    stores (and copies into the tensor-parallel peers); refused rows take
//    the warp's f32 product.  The consumers reuse a record stage only after
//    its chain warp is done with it; the data stream never waits for a chain.
// The activation row sits in shared memory in a layout that puts the lanes
// of a quarter-warp on distinct banks for both block orders.
#include <algorithm>
#include <cstdint>

#include "common.cuh"
#include "kernels.h"
#include "a8_refused.cuh"
#include "gemv_row.cuh"
#include "p2p.cuh"
#include "rms.cuh"

namespace mimgpu {

namespace {

constexpr int kCW = 16;               // consumer warps
constexpr int kCT = kCW * 32;         // consumer threads
constexpr int kNC = 2;                // chain warps
constexpr int kThreads = kCT + 32 + 32 * kNC;  // + the producer warp and the chain warps
constexpr int kMaxSB = 256;           // blocks per stage at most (two lanes per block)
constexpr int kMaxSlots = 8;
constexpr int kSmemMax = 227 * 1024;
constexpr unsigned FULL = 0xffffffffu;

struct RowParams {
    GemvSeg seg[kMaxSegs];
    int nseg;
    const float *x;     // f32 activations (refused rows)
    ActQ8 act;
    long long K;
    int nb;             // blocks per row
    int sb;             // blocks per stage: whole rows, a multiple of `unit` rows
    int unit;           // rows per 16-byte multiple of row bytes: slabs and stages come in these
    int rstages;        // stages of rows in the record ring
    int slots, slot_bytes;
    int off_act, off_hdr, off_ys, off_rec, off_bad, off_ring;
    P2P put;
    unsigned *status;
    GemvPrefetch pf;    // the next launches' weights into L2 (pf.nt 0: none)
    GemvNorm nrm;       // nrm.x set: the activation row is rms_norm(nrm.x), made here
    int off_aux;        // floats: the slab's residual values (pre_res)
    int pre_res;        // one segment with a residual: its slab's values read at the start
};

// rms_norm.v1 of the residual row and its 8-bit blocks, made by the 16
// consumer warps of every CTA in place of a separate kernel (fastRMSNorm,
// interp/fast.go:434-485, then QuantizeBlocks, q8.go:50-97): the float64
// sum of squares as a tree with the in-order fallback of rms.cuh, then per
// 256-element block (warp w takes blocks w, w + 16, ...; lane l elements
// 8l..8l+7) the normalised values, their amax and refusal, the quants in
// the act_off layout and the per-half headers.  CTA 0 writes the normalised
// row to nrm.h; refused rows recompute its elements from the residual,
// 1/rms (misc[2]) and the norm weights.  Same bits as rmsnorm_quant_kernel.
constexpr int kNormRounds = 2;  // blocks per consumer warp: K <= 2 * 16 * 256
__device__ __forceinline__ void stage_norm(const RowParams &p, uint8_t *smem, int *misc, double *red,
                                           const float (&nsc)[kNormRounds][8]) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, K = (int)p.K;
    const float *x = p.nrm.x;
    float xv[kNormRounds][8];
    double ss = 0.0;
#pragma unroll
    for (int u = 0; u < kNormRounds; u++) {
        const int kb = w + u * kCW;
        if (kb < p.nb) {
            const int e0 = kb * 256 + lane * 8;
            const float4 xa = __ldcg((const float4 *)(x + e0)), xb = __ldcg((const float4 *)(x + e0 + 4));
            xv[u][0] = xa.x; xv[u][1] = xa.y; xv[u][2] = xa.z; xv[u][3] = xa.w;
            xv[u][4] = xb.x; xv[u][5] = xb.y; xv[u][6] = xb.z; xv[u][7] = xb.w;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const double e = (double)xv[u][j];
                ss = __fma_rn(e, e, ss);  // e*e is exact in float64
            }
        }
    }
    ss = warp_sum_d(ss);
    if (lane == 0) red[w] = ss;
    asm volatile("bar.sync 2, %0;" ::"r"(kCT) : "memory");
    // the kCW partials by a butterfly over the whole warp: every level adds
    // the same two values in both lanes of a pair, so all threads get the
    // same bits
    double tot = lane < kCW ? red[lane] : 0.0;
#pragma unroll
    for (int o = 16; o; o >>= 1) tot += __shfl_xor_sync(FULL, tot, o);
    float ms;
    // a term passes through at most 8 kNormRounds products-and-sums in its
    // thread, 5 shuffle levels and kCW partials: a depth bound of K/kCT + 32
    if (!rms_mean_certain(tot, K, K / kCT + 32, ms)) {  // the same decision in every thread
        if (threadIdx.x == 0) misc[1] = __float_as_int((float)__ddiv_rn(rms_seq_sum_cg(x, K), (double)K));
        asm volatile("bar.sync 2, %0;" ::"r"(kCT) : "memory");
        ms = __int_as_float(misc[1]);
    }
    const float inv = rms_inv_of_mean(ms, p.nrm.eps);
    if (threadIdx.x == 0) misc[2] = __float_as_int(inv);  // for the f32 product of refused rows
#pragma unroll
    for (int u = 0; u < kNormRounds; u++) {
        const int kb = w + u * kCW;
        if (kb >= p.nb) break;
        const int e0 = kb * 256 + lane * 8;
        float v[8];
        float am = 0.f;
        int bad = 0;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            v[j] = __fmul_rn(xv[u][j], inv);
            if (p.nrm.scale) v[j] = __fmul_rn(v[j], nsc[u][j]);
            const float a = fabsf(v[j]);
            const bool b = !(a <= 0x1p60f);
            bad |= b;
            am = fmaxf(am, b ? 0.f : a);
        }
        if (blockIdx.x == 0) {  // one writer: the same 16 KB stored by every CTA backs up the store queue
            *(float4 *)(p.nrm.h + e0) = make_float4(v[0], v[1], v[2], v[3]);
            *(float4 *)(p.nrm.h + e0 + 4) = make_float4(v[4], v[5], v[6], v[7]);
        }
        am = warp_max(am);
        bad = __any_sync(FULL, bad);
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
        // lane pairs hold runs of 16, quads runs of 32
        const int s16 = s8 + __shfl_xor_sync(FULL, s8, 1);
        const int s32 = s16 + __shfl_xor_sync(FULL, s16, 2);
        const int c = lane >> 1, hh = c >> 3, a = c & 7;  // chunk of 16 quants, half, chunk in the half
        *(uint2 *)(smem + p.off_act + act_off(kb, hh) + 16 * a + 8 * (lane & 1)) = make_uint2(qw[0], qw[1]);
        // half hh's header (runs of 32: lanes 16hh + 4r) and sums of 16 (lanes 16hh + 2r)
        const int base = lane & 16;
        uint32_t xs2[2], ys4[4];
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const int lo = __shfl_sync(FULL, s32, base + 8 * r), hi = __shfl_sync(FULL, s32, base + 8 * r + 4);
            xs2[r] = ((uint32_t)lo & 0xFFFFu) | ((uint32_t)hi << 16);
        }
#pragma unroll
        for (int r = 0; r < 4; r++) {
            const int lo = __shfl_sync(FULL, s16, base + 4 * r), hi = __shfl_sync(FULL, s16, base + 4 * r + 2);
            ys4[r] = ((uint32_t)lo & 0xFFFFu) | ((uint32_t)hi << 16);
        }
        if ((lane & 15) == 0) {
            const int hb = 2 * kb + hh;
            *(uint4 *)(smem + p.off_hdr + hdr_off(hb)) =
                make_uint4(xs2[0], xs2[1], __float_as_uint(__fdiv_rn(am, 127.f)), bad ? 0u : 1u);
            *(uint4 *)(smem + p.off_ys + hdr_off(hb)) = make_uint4(ys4[0], ys4[1], ys4[2], ys4[3]);
        }
        if (bad && lane == 0) misc[0] = 0;
    }
}

__global__ void __launch_bounds__(kThreads, 1) gemv_row_kernel(const __grid_constant__ RowParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = (uint64_t *)smem;       // data slot landed (producer's bytes)
    uint64_t *cons = full + kMaxSlots;       // data slot read by the 16 consumer warps
    uint64_t *rdone = cons + kMaxSlots;      // record stage written by the 16 consumer warps
    uint64_t *rfree = rdone + kMaxSlots;     // record stage finished by its chain warp
    int *misc = (int *)(smem + 4 * kMaxSlots * 8);  // [0] activation row quantized
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, cta = blockIdx.x, nb = p.nb, sb = p.sb, rps = sb / nb, RS = p.rstages;
    if (threadIdx.x == 0) {
        for (int s = 0; s < p.slots; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&cons[s], kCW);
        }
        for (int s = 0; s < RS; s++) {
            mbar_init(&rdone[s], kCW);
            mbar_init(&rfree[s], 1);
        }
        misc[0] = 1;
        fence_barrier_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == kCW) {
        // ------------------------------------------------ producer (one thread)
        if (lane != 0) return;
        uint8_t *ring = smem + p.off_ring;
        int n = 0, slot = 0, ph = 0;
        bool ok = true;
        // every weight byte is read once per step: first out of L2, so the
        // activations, caches and norm weights stay
        const uint64_t pol = l2_policy_evict_first();
        for (int s = 0; s < p.nseg && ok; s++) {
            int r0, nr;
            slab(p.seg[s].n, cta, G, p.unit, r0, nr);
            const int bb = block_bytes(p.seg[s].dt);
            const int nblk = nr * nb;
            const uint8_t *src = p.seg[s].w + (long long)r0 * nb * bb;
            for (int k0 = 0; k0 < nblk; k0 += sb, n++) {
                // slot reuse: the consumers are done with the stage p.slots back
                if (n >= p.slots && !mbar_wait_bounded(&cons[slot], ph ^ 1, p.status)) {
                    ok = false;
                    break;
                }
                const uint32_t bytes = (uint32_t)(min(sb, nblk - k0) * bb);
                mbar_arrive_expect_tx(&full[slot], bytes);
                bulk_g2s_hint(ring + (size_t)slot * p.slot_bytes, src + (long long)k0 * bb, bytes, &full[slot], pol);
                if (++slot == p.slots) {
                    slot = 0;
                    ph ^= 1;
                }
            }
        }
        // the next launch's first bytes of this CTA's slabs into L2, while
        // this launch's last stages are in flight
        if (ok) slab_prefetch(p.pf, cta);
        // copies still in flight land before the block exits
        for (int u = max(0, n - p.slots); u < n; u++)
            mbar_wait_bounded(&full[u % p.slots], (u / p.slots) & 1, p.status);
        return;
    }

    // ------------------------------------------- consumers and the chain warps
    const int tid = threadIdx.x;
    // the norm weights are read-only: in registers before the wait
    float nsc[kNormRounds][8];
    if (warp < kCW && p.nrm.x) {
        const uint64_t keep = l2_policy_evict_last();
#pragma unroll
        for (int u = 0; u < kNormRounds; u++) {
            const int kb = warp + u * kCW, e0 = kb * 256 + lane * 8;
            float4 sa = make_float4(1.f, 1.f, 1.f, 1.f), sb4 = sa;
            if (kb < p.nb && p.nrm.scale) {
                sa = ldg_keep4((const float4 *)(p.nrm.scale + e0), keep);
                sb4 = ldg_keep4((const float4 *)(p.nrm.scale + e0 + 4), keep);
            }
            nsc[u][0] = sa.x; nsc[u][1] = sa.y; nsc[u][2] = sa.z; nsc[u][3] = sa.w;
            nsc[u][4] = sb4.x; nsc[u][5] = sb4.y; nsc[u][6] = sb4.z; nsc[u][7] = sb4.w;
        }
    }
    pdl_wait();
    float *aux = (float *)(smem + p.off_aux);
    if (warp < kCW && p.nrm.x) {
        stage_norm(p, smem, misc, (double *)(smem + 4 * kMaxSlots * 8 + 16), nsc);
        for (int i = tid; i < RS * rps; i += kCT) smem[p.off_bad + i] = 0;
    } else if (warp > kCW) {
        // the residual of this CTA's rows, written by an earlier kernel and
        // final once the wait above returned: read now, beside the
        // activation staging, rather than by each row chain at its end
        if (p.pre_res) {
            int r0, nr;
            slab(p.seg[0].n, cta, G, p.unit, r0, nr);
            for (int i = threadIdx.x - (kCT + 32); i < nr; i += 32 * kNC) aux[i] = __ldcg(p.seg[0].res + r0 + i);
        }
    } else if (warp < kCW) {
        // the activation row into shared memory (act_off layout), the
        // per-half headers (xs of the 4 runs of 32, dx, ok), the sums of 16
        // Every load of a thread is issued before its first store, so the
        // staging costs one round trip to L2 (the previous kernel wrote the
        // row; it is read-only from here on, hence the read-only path).
        const int nq = (int)(p.K / 16);
        constexpr int kQ = 4;  // chunks of 16 quants per thread: K <= kQ * 16 * kCT
        uint4 qv[kQ];
#pragma unroll
        for (int j = 0; j < kQ; j++) {
            const int c = tid + j * kCT;
            if (c < nq) qv[j] = __ldg((const uint4 *)(p.act.q + (long long)c * 16));
        }
        const int hb = tid, hkb = hb >> 1, hh = hb & 1;
        const bool hon = hb < 2 * nb;  // 2 nb <= 512: one half-block entry per thread at most
        uint2 xs = make_uint2(0, 0);
        uint4 ys = make_uint4(0, 0, 0, 0);
        float dx = 0.f;
        int okb = 1;
        if (hon) {
            xs = __ldg((const uint2 *)(p.act.xs + hkb * 8 + 4 * hh));
            ys = __ldg((const uint4 *)(p.act.ys + hkb * 16 + 8 * hh));
            dx = __ldg(p.act.dx + hkb);
            okb = __ldg(p.act.ok + hkb);
        }
#pragma unroll
        for (int j = 0; j < kQ; j++) {
            const int c = tid + j * kCT;
            if (c < nq) {
                const int kb = c >> 4, h = (c >> 3) & 1, a = c & 7;
                *(uint4 *)(smem + p.off_act + act_off(kb, h) + 16 * a) = qv[j];
            }
        }
        if (hon) {
            *(uint4 *)(smem + p.off_hdr + hdr_off(hb)) = make_uint4(xs.x, xs.y, __float_as_uint(dx), (unsigned)okb);
            *(uint4 *)(smem + p.off_ys + hdr_off(hb)) = ys;
            if (!okb) misc[0] = 0;  // a row is quantized when every one of its blocks is (q8.go:50-97)
        }
        for (int i = tid; i < RS * rps; i += kCT) smem[p.off_bad + i] = 0;
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kCT + 32 * kNC) : "memory");
    const bool act_ok = misc[0] != 0;
    const int rstride = (nb + 1) * 16;  // record rows padded by 16 bytes: no bank conflicts
    const uint32_t rec_s = smem_u32(smem + p.off_rec);
    uint8_t *bad = smem + p.off_bad;  // [RS * rps] rows with a non-finite block scale
    bool failed = false;              // a wait gave up: skip the work, keep the protocol

    if (warp > kCW) {
        // ------------------------------------------------ chain warps
        // Chain warp c takes the record stages m = c (mod kNC): once the
        // consumers have written them, the block-ordered chain of each row
        // (one row per lane), bias, residual, stores; refused rows take the
        // warp's f32 product.  Then the record stage is free again.
        const int c = warp - kCW - 1;
        int m = 0;
        for (int s = 0; s < p.nseg; s++) {
            const GemvSeg &sg = p.seg[s];
            int r0, nr;
            slab(sg.n, cta, G, p.unit, r0, nr);
            const int dt = sg.dt;
            const long long rb = row_bytes(dt, p.K);
            // the finished row `rel` of the slab (output row r0 + rel): bias,
            // residual, stores
            auto emit = [&](int rel, float r) {
                const int orow = r0 + rel;
                if (sg.bias) r = __fadd_rn(r, sg.bias[orow]);
                if (sg.res) r = __fadd_rn(p.pre_res ? aux[rel] : sg.res[orow], r);
                sg.y[orow] = r;
                for (int k = 0; k < (p.put.N > 1 ? p.put.N : 0); k++)
                    peer_ptr<float>(p.put, k, p.put.off)[p.put.col0 + orow] = r;
            };
            for (int lo = 0; lo < nr; lo += rps, m++) {
                if (m % kNC != c) continue;
                const int rs = m % RS;
                if (!failed && !mbar_wait_bounded(&rdone[rs], (m / RS) & 1, p.status)) failed = true;
                failed = __any_sync(FULL, failed);
                const int hi = min(nr, lo + rps);  // the stage's rows
                for (int t0 = lo; t0 < hi; t0 += 32) {
                    const int row = t0 + lane;
                    const bool valid = row < hi;
                    const int idx = rs * rps + (valid ? row - lo : 0);
                    const uint32_t rr = rec_s + (uint32_t)(idx * rstride);
                    float tot = 0.f, off = 0.f;
                    if (valid) {
                        if (dt == Q4_K) {
#pragma unroll 16
                            for (int k = 0; k < nb; k++) {
                                const uint4 v = lds128(rr + 16 * k);
                                tot = __fmaf_rn(__uint_as_float(v.x), __uint_as_float(v.y), tot);
                                off = __fmaf_rn(__uint_as_float(v.z), __uint_as_float(v.w), off);
                            }
                        } else {
#pragma unroll 16
                            for (int k = 0; k < nb; k++) {
                                const uint4 v = lds128(rr + 16 * k);
                                tot = __fmaf_rn(__uint_as_float(v.x), __uint_as_float(v.y), tot);
                            }
                        }
                    }
                    const bool refused = valid && (bad[idx] != 0 || !act_ok);
                    if (valid) bad[idx] = 0;
                    if (valid && !refused && !failed) emit(row, __fsub_rn(tot, off));
                    // rows whose weights or activations the 8-bit kernel refuses: f32 product
                    unsigned rm = __ballot_sync(FULL, refused && !failed);
                    while (rm) {
                        const int i = __ffs(rm) - 1;
                        rm &= rm - 1;
                        const int frow = r0 + t0 + i;
                        float r;
                        if (p.nrm.x) {  // the activation row exists only in this kernel: remake its elements
                            const float ninv = __int_as_float(misc[2]);
                            const float *nx = p.nrm.x, *ns = p.nrm.scale;
                            r = row_dot_f32_fn(dt, sg.w + (long long)frow * rb, nb, [&](long long e) {
                                const float v = __fmul_rn(__ldcg(nx + e), ninv);
                                return ns ? __fmul_rn(v, __ldg(ns + e)) : v;
                            });
                        } else {
                            r = row_dot_f32(dt, sg.w + (long long)frow * rb, p.x, nb);
                        }
                        if (lane == 0) emit(t0 + i, r);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&rfree[rs]);  // the record stage is free again
            }
        }
        if (p.put.N > 1) {
            // the peer stores are visible system-wide before the kernel ends
            // (the next kernel on this stream publishes the exchange)
            __syncwarp();
            if (lane == 0) __threadfence_system();
        }
        return;
    }

    // ---------------------------------------------------- consumer warps
    const uint32_t act_s = smem_u32(smem + p.off_act), hdr_s = smem_u32(smem + p.off_hdr);
    const uint32_t ys_s = smem_u32(smem + p.off_ys), ring_s = smem_u32(smem + p.off_ring);
    const int h = lane & 1;
    int m = 0, slot = 0, ph = 0, rs = 0, rph = 0;
    for (int s = 0; s < p.nseg; s++) {
        const GemvSeg &sg = p.seg[s];
        int r0, nr;
        slab(sg.n, cta, G, p.unit, r0, nr);
        const int dt = sg.dt;
        // this lane's block of every stage: the same column of every stage's rows
        const int blk = dt == Q4_K ? 16 * warp + (lane >> 1) : 8 * (16 * (warp >> 3) + (lane >> 1)) + (warp & 7);
        const bool lane_on = blk < sb;
        const int roff = blk / nb, kb = blk - roff * nb;
        const int bb = dt == Q4_K ? 144 : 210;
        const uint32_t ya = act_s + (uint32_t)act_off(lane_on ? kb : 0, h);
        const uint32_t ha = (uint32_t)hdr_off(2 * (lane_on ? kb : 0) + h);
        for (int row0 = 0; row0 < nr; row0 += rps, m++) {
            if (!failed && !mbar_wait_bounded(&full[slot], ph, p.status)) failed = true;
            // the record stage this one reuses has been chained
            if (!failed && m >= RS && !mbar_wait_bounded(&rfree[rs], rph ^ 1, p.status)) failed = true;
            failed = __any_sync(FULL, failed);
            const int row = row0 + roff;
            const bool active = !failed && lane_on && row < nr;
            int S = 0, M = 0;
            uint32_t dh = 0, mh = 0;
            float dx = 0.f;
            if (active) {
                const uint32_t ba = ring_s + (uint32_t)(slot * p.slot_bytes + blk * bb);
                if (dt == Q4_K) {
                    q4k_half(ba, h, ya, hdr_s + ha, S, M, dh, mh, dx);
                } else {
                    switch ((warp & 7) >> 1) {
                    case 0: q6k_half<0>(ba, h, ya, ys_s + ha, S, dh); break;
                    case 1: q6k_half<1>(ba, h, ya, ys_s + ha, S, dh); break;
                    case 2: q6k_half<2>(ba, h, ya, ys_s + ha, S, dh); break;
                    default: q6k_half<3>(ba, h, ya, ys_s + ha, S, dh); break;
                    }
                    dx = __uint_as_float(lds128(hdr_s + ha).z);
                }
            }
            S += __shfl_xor_sync(FULL, S, 1);
            M += __shfl_xor_sync(FULL, M, 1);
            __syncwarp();
            if (lane == 0) mbar_arrive(&cons[slot]);  // the data slot goes back to the producer
            if (active && h == 0) {
                const int idx = rs * rps + roff;
                const float d = f16f(dh);
                float fm = 0.f, pm = 0.f;
                bool nf = !f16_finite(dh);
                if (dt == Q4_K) {
                    fm = __int2float_rn(M);
                    pm = __fmul_rn(f16f(mh), dx);
                    nf |= !f16_finite(mh);
                }
                sts128(rec_s + (uint32_t)(idx * rstride + kb * 16), __float_as_uint(__int2float_rn(S)),
                       __float_as_uint(__fmul_rn(d, dx)), __float_as_uint(fm), __float_as_uint(pm));
                if (nf) bad[idx] = 1;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&rdone[rs]);
            if (++slot == p.slots) {
                slot = 0;
                ph ^= 1;
            }
            if (++rs == RS) {
                rs = 0;
                rph ^= 1;
            }
        }
    }
}

// The fewest whole rows of type dt whose bytes are a multiple of 16 (1 for
// Q4_K; 2, 4 or 8 for Q6_K rows of 210-byte blocks).
int row_unit(int dt, long long K) {
    const long long rb = row_bytes(dt, K);
    int u = 1;
    while ((rb * u) % 16) u *= 2;
    return u;
}

struct RowPlan {
    int unit, sb, rstages, slots, slot_bytes, smem;
    int off_act, off_hdr, off_ys, off_aux, off_rec, off_bad, off_ring;
    int pre_res;
};

bool plan_row(const GemvSeg *segs, int nseg, long long K, RowPlan &pl) {
    // K <= 32768: the prologue stages at most 4 chunks of 16 quants per consumer thread
    if (K % 256 || K <= 0 || K / 256 > kMaxSB || K > 4LL * 16 * kCT) return false;
    const int nb = (int)(K / 256);
    int maxbb = 0;
    for (int i = 0; i < nseg; i++) maxbb = max(maxbb, block_bytes(segs[i].dt));
    // rows per stage: whole rows, up to 256 blocks, a multiple of the unit
    // (a Q6_K row of 7, 14 or 28 blocks is not a 16-byte multiple)
    pl.unit = 1;
    for (int i = 0; i < nseg; i++) pl.unit = max(pl.unit, row_unit(segs[i].dt, K));
    const int rps = kMaxSB / nb / pl.unit * pl.unit;
    if (rps < 1) return false;
    pl.sb = rps * nb;
    auto al = [](int v, int a) { return (v + a - 1) / a * a; };
    // a slot holds the largest stage the launch has: rows per stage, or a
    // whole slab when that is smaller (a q|k|v launch's Q6_K v slab of a
    // few rows needs no full Q6_K stage), so small launches get more slots
    // and every copy is in flight from the start
    const int G = num_sms();
    long long stage_max = 16;
    for (int i = 0; i < nseg; i++) {
        const long long units = segs[i].n / pl.unit;
        const long long slab_rows = (units + G - 1) / G * pl.unit;
        stage_max = std::max(stage_max, std::min((long long)rps, slab_rows) * nb * block_bytes(segs[i].dt));
    }
    pl.slot_bytes = al((int)std::min(stage_max, (long long)pl.sb * maxbb), 128);
    int o = 512;  // barriers and flags
    pl.off_act = o;
    o = al(o + act_bytes(nb), 16);
    pl.off_hdr = o;
    o += hdr_bytes(nb);
    pl.off_ys = o;
    o += hdr_bytes(nb);
    // aux: the slab's residual values, read at the start (one matrix with a
    // residual, a few KB at most)
    long long slab_max = 0;
    for (int i = 0; i < nseg; i++) {
        const long long units = segs[i].n / pl.unit;
        slab_max = std::max(slab_max, (units + G - 1) / G * pl.unit);
    }
    pl.pre_res = nseg == 1 && segs[0].res && slab_max <= 1024;
    pl.off_aux = o;
    if (pl.pre_res) o += al((int)slab_max * 4, 16);
    pl.off_rec = o;
    const int fixed = o, rec_stage = rps * (nb + 1) * 16;
    // the most data slots first (3 at least), then the most record stages (2 at least)
    for (int slots = kMaxSlots; slots >= 3; slots--)
        for (int rst = kMaxSlots; rst >= 2; rst--) {
            int e = fixed + rst * rec_stage;
            pl.off_bad = e;
            e = al(e + rst * rps, 128);
            pl.off_ring = e;
            pl.smem = e + slots * pl.slot_bytes;
            if (pl.smem <= kSmemMax) {
                pl.slots = slots;
                pl.rstages = rst;
                return true;
            }
        }
    return false;
}

cudaError_t prepare_row() {
    static std::atomic<unsigned long long> done{0};
    return once_per_device(done, [] {
        return cudaFuncSetAttribute(gemv_row_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
    });
}

}  // namespace

bool gemv_row_ok(const GemvSeg *segs, int nseg, const ActQ8 &act, long long K) {
    if (nseg <= 0 || nseg > kMaxSegs) return false;
    for (int i = 0; i < nseg; i++)
        if ((unsigned long long)segs[i].n * (unsigned long long)num_sms() >= (1ULL << 32)) return false;
    if (((uintptr_t)act.q & 15) || ((uintptr_t)act.ys & 15) || ((uintptr_t)act.xs & 7)) return false;
    for (int i = 0; i < nseg; i++) {
        if (segs[i].dt != Q4_K && segs[i].dt != Q6_K) return false;
        if (K % 256 || ((uintptr_t)segs[i].w & 15)) return false;
    }
    RowPlan pl;
    if (!plan_row(segs, nseg, K, pl)) return false;
    // every matrix a whole number of units: its slabs and stages are 16-byte multiples
    for (int i = 0; i < nseg; i++)
        if (segs[i].n % pl.unit) return false;
    return true;
}

cudaError_t gemv_row_prepare() { return prepare_row(); }

bool gemv_prefetch_add(const GemvSeg *segs, int nseg, long long K, uint32_t bytes, GemvPrefetch &pf) {
    RowPlan pl;
    if (pf.nt >= kMaxPrefetchTargets || bytes == 0) return false;
    if (nseg <= 0 || nseg > kMaxSegs || bytes % 16 || !plan_row(segs, nseg, K, pl)) return false;
    GemvPrefetchTarget t{};
    for (int i = 0; i < nseg; i++) {
        if ((segs[i].dt != Q4_K && segs[i].dt != Q6_K) || ((uintptr_t)segs[i].w & 15) || segs[i].n % pl.unit ||
            (unsigned long long)segs[i].n * (unsigned long long)num_sms() >= (1ULL << 32))
            return false;
        t.w[i] = segs[i].w;
        t.n[i] = segs[i].n;
        t.dt[i] = segs[i].dt;
    }
    t.nseg = nseg;
    t.unit = pl.unit;
    t.K = K;
    t.bytes = bytes;
    pf.t[pf.nt++] = t;
    pf.G = num_sms();
    return true;
}

cudaError_t launch_gemv_row(const GemvSeg *segs, int nseg, const float *x, ActQ8 act, long long K, unsigned *status,
                            cudaStream_t st, bool pdl, const P2P *put, const GemvPrefetch *pf, const GemvNorm *nrm) {
    RowPlan pl;
    if (!plan_row(segs, nseg, K, pl)) return cudaErrorInvalidValue;
    cudaError_t e = prepare_row();
    if (e != cudaSuccess) return e;
    RowParams p = {};
    for (int i = 0; i < nseg; i++) p.seg[i] = segs[i];
    p.nseg = nseg;
    p.x = x;
    p.act = act;
    p.K = K;
    p.nb = (int)(K / 256);
    p.sb = pl.sb;
    p.unit = pl.unit;
    p.rstages = pl.rstages;
    p.slots = pl.slots;
    p.slot_bytes = pl.slot_bytes;
    p.off_act = pl.off_act;
    p.off_hdr = pl.off_hdr;
    p.off_ys = pl.off_ys;
    p.off_aux = pl.off_aux;
    p.pre_res = pl.pre_res;
    p.off_rec = pl.off_rec;
    p.off_bad = pl.off_bad;
    p.off_ring = pl.off_ring;
    if (put) p.put = *put;
    if (pf) p.pf = *pf;
    if (nrm) {
        // 16-byte aligned rows; the in-order fallback and the staging read K floats
        if (!nrm->x || !nrm->h || ((uintptr_t)nrm->x & 15) || ((uintptr_t)nrm->h & 15) ||
            ((uintptr_t)nrm->scale & 15) || nrm->h != x)
            return cudaErrorInvalidValue;
        if (p.nb > kNormRounds * kCW) return cudaErrorInvalidValue;
        p.nrm = *nrm;
    }
    p.status = status;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3(num_sms());
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = (size_t)pl.smem;
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemv_row_kernel, p);
}

}  // namespace mimgpu
