// k_step.cu -- the whole one-token decode step of the llama graph
// (importer/llama.go:400-534 of gsoultan/mimir-model; one Session.Run of
// interp/interp.go:409-526 at T = 1) as ONE persistent kernel on sm_100a.
//
// Why: a decode token streams every weight once (4.9 GB at the 8B shape)
// and does almost nothing else, but as ~290 dependent kernels each launch
// pays a ramp to its first bytes and a tail, and the small kernels between
// the products leave HBM idle.  Here one CTA per SM lives for the whole
// step, and its producer thread streams the CTA's share of every matrix of
// every layer, in order, through one ring of shared memory: it runs ahead
// across op boundaries while the rest of the CTA waits for the activations
// the next product needs, so the weight stream does not stop at a
// dependency.
//
// Roles in a CTA (608 threads):
//   * producer (warp 16, one thread): one cp.async.bulk per stage of whole
//     rows (two for the paired gate|up stages) into a byte ring of up to 8
//     stages in flight; a stage's bytes are reused once the consumers have
//     read it.
//   * consumers (warps 0-15): before each product the activation row, in
//     8-bit blocks, goes into shared memory -- by RMSNorm + quantization
//     computed by every CTA for itself (q|k|v, gate|up, head), or staged from
//     the blocks the attention units or the SwiGLU quantizers wrote (o,
//     down); then one half block per lane per stage, the exact int32 sums of
//     dotQ8KRef (gemv_row.cuh), records to the chain warps.  The consumers
//     of the first CTAs also run the attention units.
//   * chain warps (warps 17, 18; alternate stages): each row's block-ordered
//     float chain (internal/kernels/q8k_test.go:35-117) and the op's
//     epilogue: RoPE and the f16 cache write (q|k|v), the residual add (o,
//     down), SiLU(gate) * up and the 8-bit blocks of the SwiGLU output
//     (gate|up), logits and the greedy key (head).
// Ops that need every CTA's output first (attention after q|k|v, o after
// attention, ...) wait on grid counters: a CTA adds to a counter once its
// share is written (release), the waiters poll it (acquire) against
// arrivals x (steps completed + 1), so nothing is ever reset.  Every wait is
// bounded; a wait that runs out sets DEV_TIMEOUT in the status word and the
// kernel finishes without waiting again.
//
// Every value is bit-identical to the kernel-per-op path: the same block
// sums, chains, attention arithmetic (amd64_math.cuh) and rounding steps.
#include <cstdint>

#include "a8_refused.cuh"
#include "amd64_math.cuh"
#include "common.cuh"
#include "gemv_row.cuh"
#include "kernels.h"
#include "rms.cuh"
#include "step.h"

namespace mimgpu {
namespace {

constexpr int kCW = 16;                         // consumer warps
constexpr int kCT = kCW * 32;                   // consumer threads
constexpr int kNC = 2;                          // chain warps
constexpr int kThreads = kCT + 32 + 32 * kNC;   // 608
constexpr int kStg = 16;                        // data stages in flight at most
constexpr int kRS = 4;                          // record stages
constexpr int kMaxSB = 256;                     // blocks per stage (one half block per consumer lane)
constexpr int kRowsCap = 32;                    // rows per stage at most (K >= 2048)
constexpr int kRecStage = 4608;                 // bytes of a record stage: rows * (nb + 1) * 16 <= 4608
constexpr int kSmem = 227 * 1024;
constexpr int kMaxK = 4 * 16 * kCT;             // activation staging: 4 chunks of 16 quants per thread
constexpr int kMaxE = 2 * 256 * kCW;            // RMSNorm: two 256-element blocks per consumer warp
constexpr unsigned FULLM = 0xffffffffu;
constexpr int kRoles = 1 + kCW + kNC;

enum { J_QKV = 0, J_O = 1, J_GU = 2, J_DOWN = 3, J_HEAD = 4 };
// grid counters: [0] embedding, then 5 per layer, then the SwiGLU blocks
enum { C_QKV = 0, C_ATT = 1, C_O = 2, C_QUANT = 3, C_DOWN = 4 };

struct Smem {
    int off_lt, off_act, off_hdr, off_ys, off_rec, off_bad, off_ring, ring;
};

// misc words after the barriers
constexpr int kMiscOff = 512;  // after the barriers: 2 x kStg + 2 x kRS mbarriers
struct Misc {
    int act_ok;
    int roles_done;
    int abort;
    unsigned qmask;   // SwiGLU blocks this CTA completes (chain warps)
    float inv[4];     // rms inverse of the job's activation (refused rows recompute it)
    float hmax[8], hsum[8];
    float red[16][8];
    float2 rope[64];  // cos / sin of the step's position (chain warps)
};

__device__ __forceinline__ unsigned ld_acq(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_rel(unsigned *p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned atom_acqrel(unsigned *p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ void bar_cons() { asm volatile("bar.sync 1, %0;" ::"r"(kCT) : "memory"); }
__device__ __forceinline__ void bar_chain() { asm volatile("bar.sync 2, %0;" ::"r"(32 * kNC) : "memory"); }

__device__ __forceinline__ uint64_t wait_limit(const unsigned *status) { return dev_wait_limit(status); }

// A wait of this CTA gave up: later waits return at once.
__device__ __forceinline__ bool aborted(const Misc &ms) { return *(volatile const int *)&ms.abort != 0; }
__device__ __forceinline__ void set_abort(Misc &ms) { *(volatile int *)&ms.abort = 1; }

// Polls a grid counter until it reaches `target` (wrap-safe).  One thread.
// Gives up at the wait limit, or at once when another wait of the kernel
// already gave up (the status word says so), setting misc.abort.

__device__ bool grid_wait(const unsigned *ctr, unsigned target, unsigned *status, Misc &ms) {
    if (aborted(ms)) return false;
    if ((int)(ld_acq(ctr) - target) >= 0) return true;
    const uint64_t t0 = global_ns(), lim = wait_limit(status);
    for (uint32_t i = 1;; i++) {
        if ((int)(ld_acq(ctr) - target) >= 0) return true;
        if ((i & 63) == 0) {
            if (*(volatile unsigned *)status & DEV_TIMEOUT) break;
            if (global_ns() - t0 > lim) {
                atomicOr(status, (unsigned)DEV_TIMEOUT);
                break;
            }
        }
    }
    set_abort(ms);
    return false;
}

__device__ __forceinline__ bool mbar_wait_s(uint64_t *bar, uint32_t parity, unsigned *status, Misc &ms) {
    if (mbar_try_wait(bar, parity)) return true;
    if (aborted(ms)) return false;
    const uint64_t t0 = global_ns(), lim = wait_limit(status);
    for (uint32_t i = 1;; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255) == 0) {
            if (aborted(ms)) return false;
            if (global_ns() - t0 > lim) break;
        }
    }
    atomicOr(status, (unsigned)DEV_TIMEOUT);
    set_abort(ms);
    return false;
}

// Timeline stamp (profiling sessions only).
__device__ __forceinline__ void stamp(const StepParams &p, int slot) {
    if (p.trace) p.trace[(size_t)blockIdx.x * step_trace_cta_words(p.L) + slot] = global_ns();
}
// CTA 0's per-stage log (profiling sessions only)
__device__ __forceinline__ void stage_stamp(const StepParams &p, int m, int k) {
    if (p.trace && blockIdx.x == 0 && m < kStageLog)
        p.trace[(size_t)gridDim.x * step_trace_cta_words(p.L) + 4 * m + k] = global_ns();
}
__device__ __forceinline__ int jslot(int j, int k) { return 2 + 16 * j + k; }

// ------------------------------------------------------------ the jobs
// One segment of a job: a weight matrix cut into slabs of rows across the
// CTAs, or (kv) the key or value rows of one attention unit's kv head,
// streamed whole to the CTA that runs the unit.
struct Seg {
    const uint8_t *w, *w2;  // the matrix; w2: the up matrix of a paired gate|up stage
    int dt, n, nb, bb, unit, rps;
    int rb;
    int kv;                 // 1: key / value rows of an attention unit (no records, no chain)
};

// Attention units: HU query heads of one kv head each, one per CTA of the
// first `units` CTAs.
__device__ __forceinline__ int attn_hu(const StepParams &p) { return 2; }  // H / Hkv is even (step_ok)
__device__ __forceinline__ int attn_units(const StepParams &p) { return p.H / attn_hu(p); }

constexpr int kKvRows = 64;  // keys per key / value stage (16 KB)

__device__ __forceinline__ int njobs(const StepParams &p) { return 4 * p.L + 1; }
// q|k|v: q, k, v; o: the unit's keys, its values, o; others one matrix
__device__ __forceinline__ int nsegs(int kind) { return kind == J_QKV || kind == J_O ? 3 : 1; }

// The rows of segment g this CTA takes: a slab of the matrix, or every key
// of its attention unit.
__device__ __forceinline__ void seg_rows(const Seg &g, int cta, int G, int &r0, int &nr) {
    if (g.kv) {
        r0 = 0;
        nr = g.n;
        return;
    }
    slab(g.n, cta, G, g.unit, r0, nr);
}

// nk: keys of this step (position + 1)
__device__ Seg get_seg(const StepParams &p, const StepLayer *lt, int job, int s, int nk) {
    const int kind = job == 4 * p.L ? J_HEAD : job & 3;
    Seg g;
    g.w2 = nullptr;
    g.kv = 0;
    int K = p.E;
    if (kind == J_O && s < 2) {
        const int unit = blockIdx.x;
        const bool mine = unit < attn_units(p);
        const int kvh = mine ? unit * attn_hu(p) / (p.H / p.Hkv) : 0;
        const StepLayer &ly = lt[job >> 2];
        g.w = (const uint8_t *)(s == 0 ? ly.kc : ly.vc) + (size_t)kvh * p.C * p.D * 2;
        g.dt = F16;
        g.n = mine ? nk : 0;
        g.nb = 0;
        g.bb = 0;
        g.rb = p.D * 2;
        g.unit = 1;
        g.rps = kKvRows;
        g.kv = 1;
        return g;
    }
    if (kind == J_HEAD) {
        g.w = p.head;
        g.dt = p.head_dt;
        g.n = p.V;
    } else {
        const StepLayer &ly = lt[job >> 2];
        const int i = kind == J_QKV ? s : kind == J_O ? 3 : kind == J_GU ? 4 : 6;  // (o is segment 2)
        g.w = ly.w[i];
        g.dt = ly.dt[i];
        g.n = kind == J_QKV ? (s == 0 ? p.E : p.Hkv * p.D) : kind == J_GU ? p.F : p.E;
        if (kind == J_GU) g.w2 = ly.w[5];
        if (kind == J_DOWN) K = p.F;
    }
    g.nb = K / 256;
    g.bb = g.dt == Q4_K ? 144 : 210;
    g.rb = g.nb * g.bb;
    int u = 1;
    while ((g.rb * u) & 15) u <<= 1;
    if (kind == J_QKV && s < 2 && u < 2) u = 2;  // RoPE pairs stay in one slab and one stage
    g.unit = u;
    g.rps = (kMaxSB / g.nb / (g.w2 ? 2 : 1)) / u * u;
    return g;
}

// A position in the CTA's sequence of weight stages (job, segment, stage).
struct Cursor {
    int j, s, row0, r0, nr;
    Seg g;
};
__device__ __forceinline__ int kind_of(const StepParams &p, int j) { return j == 4 * p.L ? J_HEAD : j & 3; }
__device__ void cur_fix(Cursor &c, const StepParams &p, const StepLayer *lt, int nj, int nk) {
    while (c.j < nj && c.row0 >= c.nr) {
        c.row0 = 0;
        if (++c.s >= nsegs(kind_of(p, c.j))) {
            c.s = 0;
            if (++c.j >= nj) break;
        }
        c.g = get_seg(p, lt, c.j, c.s, nk);
        seg_rows(c.g, blockIdx.x, gridDim.x, c.r0, c.nr);
    }
}
__device__ void cur_start(Cursor &c, const StepParams &p, const StepLayer *lt, int nj, int nk) {
    c.j = c.s = c.row0 = 0;
    c.g = get_seg(p, lt, 0, 0, nk);
    seg_rows(c.g, blockIdx.x, gridDim.x, c.r0, c.nr);
    cur_fix(c, p, lt, nj, nk);
}
__device__ __forceinline__ void cur_step(Cursor &c, const StepParams &p, const StepLayer *lt, int nj, int nk) {
    c.row0 += c.g.rps;
    cur_fix(c, p, lt, nj, nk);
}

// Next stage's ring offset (producer and consumers compute the same sequence).
__device__ __forceinline__ uint32_t ring_next(uint32_t &head, uint32_t bytes, uint32_t ring) {
    const uint32_t off = head + bytes <= ring ? head : 0u;
    head = off + bytes;
    return off;
}

// ---------------------------------------- 8-bit blocks of one 256-element block
// RoundToEven(127 v / am) computed in float64, as QuantizeBlocks does
// (q8.go:50-97).  The f32 quotient y = RN(RN(127 v) / am) is within 2^-16 of
// the exact one (|127 v / am| <= 127, two roundings), so rintf(y) is the
// float64 result unless y lies within 2^-15 of a half-integer (or am is so
// small that 127 v loses bits); those take the float64 division.
__device__ __forceinline__ int quant_q(float v, float am) {
    const float y = __fdiv_rn(__fmul_rn(v, 127.f), am);
    if (am >= 0x1p-100f && fabsf(__fsub_rn(__fsub_rn(y, floorf(y)), 0.5f)) > 0x1p-12f) return (int)rintf(y);
    return (int)rint(__ddiv_rn(127.0 * (double)v, (double)am));
}

// Lane l holds elements 8l..8l+7 of the block.  QuantizeBlocks
// (internal/kernels/q8.go:50-97): amax, refusal of NaN / Inf / |x| > 2^60,
// q = RoundToEven(127 x / amax) in float64, dx = amax / 127; s16 / s32 are
// the sums of the lane's run of 16 / 32 (valid in lanes 2i / 4i).
__device__ __forceinline__ void warp_quant(const float (&v)[8], int (&q)[8], int &s16, int &s32, float &dx,
                                           bool &ok) {
    float am = 0.f;
    bool bad = false;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const float a = fabsf(v[i]);
        const bool b = !(a <= 0x1p60f);
        bad |= b;
        am = fmaxf(am, b ? 0.f : a);
    }
    am = warp_max(am);
    bad = __any_sync(FULLM, bad);
    int s = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        q[i] = (am != 0.f && !bad) ? quant_q(v[i], am) : 0;
        s += q[i];
    }
    s16 = s + __shfl_xor_sync(FULLM, s, 1);
    s32 = s16 + __shfl_xor_sync(FULLM, s16, 2);
    dx = __fdiv_rn(am, 127.f);
    ok = !bad;
}

__device__ __forceinline__ uint2 pack8(const int (&q)[8]) {
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        lo |= (uint32_t)(q[i] & 0xFF) << (8 * i);
        hi |= (uint32_t)(q[4 + i] & 0xFF) << (8 * i);
    }
    return make_uint2(lo, hi);
}

// The block's 8-bit data into global ActQ8 (row 0, block kb).
__device__ __forceinline__ void quant_store_global(const ActQ8 &a, int kb, const int (&q)[8], int s16, int s32,
                                                   float dx, bool ok) {
    const int lane = threadIdx.x & 31;
    __stcg((uint2 *)(a.q + (long long)kb * 256 + 8 * lane), pack8(q));
    if ((lane & 1) == 0) __stcg(a.ys + kb * 16 + (lane >> 1), (int16_t)s16);
    if ((lane & 3) == 0) __stcg(a.xs + kb * 8 + (lane >> 2), (int16_t)s32);
    if (lane == 0) {
        __stcg(a.dx + kb, dx);
        __stcg(a.ok + kb, ok ? 1 : 0);
    }
}

// The block's 8-bit data straight into the shared-memory activation layout.
__device__ __forceinline__ void quant_store_smem(uint8_t *smem, const Smem &sm, int kb, const int (&q)[8], int s16,
                                                 int s32, float dx, bool ok) {
    const int lane = threadIdx.x & 31, h = lane >> 4, hb = 2 * kb + h;
    *(uint2 *)(smem + sm.off_act + act_off(kb, h) + 8 * (lane & 15)) = pack8(q);
    if ((lane & 1) == 0) *(int16_t *)(smem + sm.off_ys + hdr_off(hb) + 2 * ((lane & 15) >> 1)) = (int16_t)s16;
    if ((lane & 3) == 0) *(int16_t *)(smem + sm.off_hdr + hdr_off(hb) + 2 * ((lane & 15) >> 2)) = (int16_t)s32;
    if ((lane & 15) == 0) {
        *(float *)(smem + sm.off_hdr + hdr_off(hb) + 8) = dx;
        *(int *)(smem + sm.off_hdr + hdr_off(hb) + 12) = ok ? 1 : 0;
    }
}

// ----------------------------------------------------- consumer pre-phases

// rms_norm of the residual (fast.go:434-485, mean bit-exact: rms.cuh) times
// the norm weight, quantized block by block into shared memory.  Every CTA
// computes the whole row for itself.  Consumer threads only.
// The wait for the residual (grid counter wctr at target) happens in here,
// after the norm weights, which are constant, are already on their way.
__device__ void norm_phase(const StepParams &p, const float *__restrict__ wn, uint8_t *smem, const Smem &sm,
                           Misc &ms, int slot, const unsigned *wctr, unsigned target, int ready_slot) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nblk = p.E / 256, bpw = (nblk + kCW - 1) / kCW;  // blocks per warp
    constexpr int kBpw = kMaxE / 256 / kCW;                     // blocks per warp at most
    float4 wreg[2 * kBpw];
#pragma unroll
    for (int j = 0; j < kBpw; j++) {
        const int kb = warp + kCW * j;
        if (j < bpw && kb < nblk) {
            wreg[2 * j] = __ldg((const float4 *)(wn + kb * 256 + 8 * lane));
            wreg[2 * j + 1] = __ldg((const float4 *)(wn + kb * 256 + 8 * lane) + 1);
        }
    }
    if (threadIdx.x == 0) {
        grid_wait(wctr, target, p.status, ms);
        stamp(p, ready_slot);
    }
    bar_cons();
    double ss = 0.0;
    for (int j = 0; j < bpw; j++) {
        const int kb = warp + kCW * j;
        if (kb < nblk) {
            const float4 *src = (const float4 *)(p.x + kb * 256 + 8 * lane);
            const float4 v0 = __ldcg(src), v1 = __ldcg(src + 1);
            const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
            for (int i = 0; i < 8; i++) ss = __fma_rn((double)v[i], (double)v[i], ss);
        }
    }
    ss = warp_sum_d(ss);
    double *dred = (double *)ms.red;  // 16 doubles
    if (lane == 0) dred[warp] = ss;
    bar_cons();
    if (threadIdx.x == 0) {
        double tot = 0.0;
#pragma unroll
        for (int i = 0; i < kCW; i++) tot += dred[i];
        float mean;
        if (!rms_mean_certain(tot, p.E, 8 * bpw + 5 + kCW, mean))
            mean = (float)__ddiv_rn(rms_seq_sum_cg(p.x, p.E), (double)p.E);
        ms.inv[slot] = rms_inv_of_mean(mean, p.eps);
        ms.act_ok = 1;
    }
    bar_cons();
    const float inv = ms.inv[slot];
    bool all_ok = true;
#pragma unroll
    for (int j = 0; j < kBpw; j++) {
        const int kb = warp + kCW * j;
        if (j >= bpw || kb >= nblk) break;
        const int e0 = kb * 256 + 8 * lane;
        const float4 *src = (const float4 *)(p.x + e0);
        const float4 v0 = __ldcg(src), v1 = __ldcg(src + 1);
        const float4 w0 = wreg[2 * j], w1 = wreg[2 * j + 1];
        const float xv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = __fmul_rn(__fmul_rn(xv[i], inv), wv[i]);
        int q[8], s16, s32;
        float dx;
        bool ok;
        warp_quant(v, q, s16, s32, dx, ok);
        quant_store_smem(smem, sm, kb, q, s16, s32, dx, ok);
        all_ok &= ok;
    }
    if (!all_ok && lane == 0) ms.act_ok = 0;  // a row is quantized when all its blocks are
    bar_cons();
}

// The 8-bit blocks another phase wrote to global memory (this step) into
// shared memory.  Consumer threads only.
__device__ void stage_phase(const ActQ8 &act, int K, uint8_t *smem, const Smem &sm, Misc &ms) {
    const int tid = threadIdx.x, nq = K / 16, nb = K / 256;
    constexpr int kQ = kMaxK / (16 * kCT);
    uint4 qv[kQ];
#pragma unroll
    for (int j = 0; j < kQ; j++) {
        const int c = tid + j * kCT;
        if (c < nq) qv[j] = __ldcg((const uint4 *)(act.q + (long long)c * 16));
    }
    const int hb = tid, hkb = hb >> 1, hh = hb & 1;
    if (tid == 0) ms.act_ok = 1;
    bar_cons();  // act_ok reset before anyone clears it
    for (int h0 = 0; h0 < 2 * nb; h0 += kCT) {
        const int hb2 = h0 + hb, k2 = hb2 >> 1;
        if (hb2 < 2 * nb) {
            const uint2 xs = __ldcg((const uint2 *)(act.xs + k2 * 8 + 4 * hh));
            const uint4 ys = __ldcg((const uint4 *)(act.ys + k2 * 16 + 8 * hh));
            const float dx = __ldcg(act.dx + k2);
            const int okb = __ldcg(act.ok + k2);
            *(uint4 *)(smem + sm.off_hdr + hdr_off(hb2)) = make_uint4(xs.x, xs.y, __float_as_uint(dx), (unsigned)okb);
            *(uint4 *)(smem + sm.off_ys + hdr_off(hb2)) = ys;
            if (!okb) ms.act_ok = 0;
        }
    }
    (void)hkb;
#pragma unroll
    for (int j = 0; j < kQ; j++) {
        const int c = tid + j * kCT;
        if (c < nq) {
            const int kb = c >> 4, h = (c >> 3) & 1, a = c & 7;
            *(uint4 *)(smem + sm.off_act + act_off(kb, h) + 16 * a) = qv[j];
        }
    }
    bar_cons();
}

// Layout of the attention scratch (the activation + record regions, free
// while attention runs): q [HU][128], outputs [HU * 128], scores [HU][n].
__host__ __device__ inline int attn_scratch_bytes(int HU, int n) { return (2 * HU * 128 + HU * n) * 4; }

// One attention unit: query heads h0..h0+HU-1 (one kv head) of the step's
// token over its nk keys [0, pos] of the f16 cache, exactly as attendRow
// (interp/fast.go:728-751) with the reference's amd64 kernels: scores in the
// eight-lane orders of scoresF16AVX2, ExpSumF32 (Cephes expf below n&~7,
// float64 exp above, its lane-sum order), the key-ordered fused weighted sum
// of wsumF16AVX2, o = acc / sum; then the 8-bit blocks of the unit's
// outputs.  The kv head's key rows, then its value rows, are stages of this
// CTA's weight stream (segments 0 and 1 of the o job), so the producer has
// loaded them while the CTA was busy with q|k|v; the token's own key and
// value rows, written this step by other CTAs, are read through L2 and
// patched into their stage.  m / head: the consumers' stage counter and
// ring offset, advanced past the stages read here.
__device__ void attn_unit(const StepParams &p, int l, int unit, int HU, int nk, uint8_t *smem, const Smem &sm,
                          Misc &ms, uint8_t *ring, uint64_t *full, uint64_t *cons, int &m, uint32_t &head, int tj) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int D = 128, G = p.H / p.Hkv, h0 = unit * HU, kvh = h0 / G;
    const int n = nk, pos = nk - 1, n4 = n & ~3, n8 = n >= 8 ? (n & ~7) : 0;
    float *q = (float *)(smem + sm.off_act);  // [HU][128]
    float *obuf = q + HU * D;                 // [HU * 128]
    float *sc = obuf + HU * D;                // [HU][n]
    for (int i = tid; i < HU * D; i += kCT) q[i] = __ldcg(p.qh + h0 * D + i);
    const uint8_t *own[2] = {(const uint8_t *)p.layers[l].kc, (const uint8_t *)p.layers[l].vc};
    // the next stage of keys (part 0) or values (part 1): wait, patch row pos
    auto land = [&](int part, int j0, int rows) -> const uint8_t * {
        const uint32_t off = ring_next(head, (uint32_t)(rows * D * 2), (uint32_t)sm.ring);
        mbar_wait_s(&full[m % kStg], (m / kStg) & 1, p.status, ms);
        uint8_t *chunk = ring + off;
        if (pos < j0 + rows) {
            if (tid < 16) {
                const uint8_t *src = own[part] + ((size_t)kvh * p.C + pos) * D * 2;
                *(uint4 *)(chunk + (pos - j0) * D * 2 + tid * 16) = __ldcg((const uint4 *)src + tid);
                // generic writes into a slot the producer's bulk copies reuse
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            }
        }
        bar_cons();
        return chunk;
    };
    auto done = [&]() {  // every warp is done with the stage
        __syncwarp();
        if (lane == 0) mbar_arrive(&cons[m % kStg]);
        m++;
    };
    // scores: a warp takes one key at a time; lane = (head hq, reference lane
    // l8), so the 32 lanes read one 16-byte piece of the key row together
    // (a broadcast) and each lane keeps its 16 q values in registers
    // (4 / HU keys per warp at a time: lane = (key kk, head hq, lane l8))
    const int l8 = lane & 7, hq = (lane >> 3) % HU, kk = lane / (8 * HU), kpw = 4 / HU;
    bar_cons();  // q in shared memory
    float qreg[16];
#pragma unroll
    for (int c8 = 0; c8 < 16; c8++) qreg[c8] = q[hq * D + 8 * c8 + l8];
    float mx = -INFINITY;
    for (int j0 = 0; j0 < n; j0 += kKvRows) {
        const int rows = min(kKvRows, n - j0);
        const uint8_t *chunk = land(0, j0, rows);
        if (j0 == 0 && tid == 0) stamp(p, jslot(tj, 9));
        for (int jb = warp * kpw; jb < rows; jb += kCW * kpw) {
            const int jj = jb + kk, jr = min(jj, rows - 1);  // past the last key: a valid row, result unused
            const uint16_t *kr = (const uint16_t *)(chunk + jr * D * 2);
            float acc = 0.f;
#pragma unroll
            for (int c8 = 0; c8 < 16; c8++) acc = __fmaf_rn(qreg[c8], h2f_bits(kr[8 * c8 + l8]), acc);
            const int j = j0 + jj;
            const float sv = __fmul_rn(score_combine(acc, j >= n4), p.scale);
            if (l8 == 0 && jj < rows) {
                sc[hq * n + j] = sv;
                mx = fmaxf(mx, sv);
            }
        }
        done();
    }
    // per-head maximum: lanes with l8 == 0 hold their head's
    if (l8 == 0) ms.red[warp][lane >> 3] = mx;
    bar_cons();
    if (tid == 0) stamp(p, jslot(tj, 10));
    if (tid < HU) {
        float mm = -INFINITY;
        for (int w = 0; w < kCW; w++)
            for (int g = tid; g < 4; g += HU) mm = fmaxf(mm, ms.red[w][g]);
        ms.hmax[tid] = mm;
    }
    bar_cons();
    for (int i = tid; i < HU * n; i += kCT) {
        const int hh = i / n, j = i - hh * n;
        const float x = __fsub_rn(sc[i], ms.hmax[hh]);
        sc[i] = j < n8 ? expf_amd64(x) : (float)exp((double)x);
    }
    bar_cons();
    if (tid < 8 * HU) {  // ExpSumF32's eight lane sums, each in key order
        const int hh = tid >> 3, l8 = tid & 7;
        float sl = 0.f;
        for (int j = l8; j < n8; j += 8) sl = __fadd_rn(sl, sc[hh * n + j]);
        ms.red[hh][l8] = sl;
    }
    bar_cons();
    if (tid < HU) {
        const float *r = ms.red[tid];
        float sum = 0.f;
        if (n8) sum = __fadd_rn(__fadd_rn(__fadd_rn(r[0], r[4]), __fadd_rn(r[1], r[5])),
                                __fadd_rn(__fadd_rn(r[2], r[6]), __fadd_rn(r[3], r[7])));
        for (int j = n8; j < n; j++) sum = __fadd_rn(sum, sc[tid * n + j]);
        ms.hsum[tid] = sum;
        if (tid == 0) stamp(p, jslot(tj, 11));
    }
    // weighted sum of the values, one fused multiply-add per key in key
    // order: warp hh (< HU) takes head hh, lane dq its head elements
    // 4dq..4dq+3 (four independent chains, 8-byte reads)
    // (warps 0-3: head warp / (4 / HU), HU elements per lane)
    const int hh = warp / (4 / HU), d0 = (warp % (4 / HU)) * 32 * HU + HU * lane;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int j0 = 0; j0 < n; j0 += kKvRows) {
        const int rows = min(kKvRows, n - j0);
        const uint8_t *chunk = land(1, j0, rows);
        if (warp < 4) {
            const float *e = sc + hh * n + j0;
            if (HU == 4) {
#pragma unroll 4
                for (int jj = 0; jj < rows; jj++) {
                    const uint2 v = *(const uint2 *)(chunk + jj * D * 2 + 2 * d0);
                    const float ev = e[jj];
                    acc[0] = __fmaf_rn(ev, h2f_bits(v.x & 0xFFFFu), acc[0]);
                    acc[1] = __fmaf_rn(ev, h2f_bits(v.x >> 16), acc[1]);
                    acc[2] = __fmaf_rn(ev, h2f_bits(v.y & 0xFFFFu), acc[2]);
                    acc[3] = __fmaf_rn(ev, h2f_bits(v.y >> 16), acc[3]);
                }
            } else {
#pragma unroll 4
                for (int jj = 0; jj < rows; jj++) {
                    const uint32_t v = *(const uint32_t *)(chunk + jj * D * 2 + 2 * d0);
                    const float ev = e[jj];
                    acc[0] = __fmaf_rn(ev, h2f_bits(v & 0xFFFFu), acc[0]);
                    acc[1] = __fmaf_rn(ev, h2f_bits(v >> 16), acc[1]);
                }
            }
        }
        done();
    }
    if (warp < 4)
        for (int i = 0; i < HU; i++) {
            const float o = __fdiv_rn(acc[i], ms.hsum[hh]);
            obuf[hh * D + d0 + i] = o;
            __stcg(p.att + (h0 + hh) * D + d0 + i, o);
        }
    bar_cons();
    if (tid == 0) stamp(p, jslot(tj, 12));
    // the unit's 8-bit blocks (HU * 128 / 256 of them), one warp each
    if (warp < HU * D / 256) {
        const int kb = (h0 * D) / 256 + warp;
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = obuf[warp * 256 + 8 * lane + i];
        int qq[8], s16, s32;
        float dx;
        bool ok;
        warp_quant(v, qq, s16, s32, dx, ok);
        quant_store_global(p.actE, kb, qq, s16, s32, dx, ok);
    }
}

// The CTA's last role to finish counts the CTA out; the last CTA of the grid
// marks the step complete, which moves every counter's target on.
__device__ __forceinline__ void role_done(const StepParams &p, Misc &ms, unsigned ep) {
    __threadfence_block();
    if (atomicAdd(&ms.roles_done, 1) != kRoles - 1) return;
    __threadfence();
    const unsigned old = atom_acqrel(p.epoch + 1, 1u);
    if (old + 1u == gridDim.x * (ep + 1)) {
        __threadfence();
        *(volatile unsigned *)p.epoch = ep + 1;
    }
}

// ------------------------------------------------------------ the kernel
__global__ void __launch_bounds__(kThreads, 1) step_kernel(const __grid_constant__ StepParams p,
                                                           const __grid_constant__ Smem sm) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = (uint64_t *)smem;
    uint64_t *cons = full + kStg;
    uint64_t *rdone = cons + kStg;
    uint64_t *rfree = rdone + kRS;
    Misc &ms = *(Misc *)(smem + kMiscOff);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    const unsigned ep = __ldcg(p.epoch);  // steps completed: grid counters aim at arrivals x (ep + 1)
    const int nk = (int)__ldcg(p.pos) + 1;  // keys of this step's attention
    const int nj = njobs(p);
    unsigned *ctr = p.sync;               // [0] embedding, [1 + 5 l + c] layer counters
    unsigned *blkctr = p.sync + 1 + 5 * p.L;  // [l][F / 256] SwiGLU block rows
    const int nfb = p.F / 256;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStg; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&cons[s], kCW);
        }
        for (int s = 0; s < kRS; s++) {
            mbar_init(&rdone[s], kCW);
            mbar_init(&rfree[s], 1);
        }
        ms.act_ok = 1;
        ms.roles_done = 0;
        ms.abort = 0;
        fence_barrier_init();
    }
    for (int i = threadIdx.x; i < kRS * kRowsCap; i += kThreads) smem[sm.off_bad + i] = 0;
    // the layer table in shared memory: every role reads it at each op
    StepLayer *lt = (StepLayer *)(smem + sm.off_lt);
    for (int i = threadIdx.x; i < p.L * (int)(sizeof(StepLayer) / 8); i += kThreads)
        ((uint2 *)lt)[i] = __ldg((const uint2 *)p.layers + i);
    __syncthreads();
    uint8_t *ring = smem + sm.off_ring;

    if (warp == kCW) {
        // -------------------------------------------------- producer
        // Stages go into the shared-memory ring in order.  The ring copies
        // mark their lines evict-first: they are read once.  (Prefetching the
        // stages after them into L2 as well was measured slower: 2.83 vs
        // 2.55 ms per 8B token; the prefetch traffic delays the
        // latency-bound loads of the small ops.)
        if (lane == 0) {
            uint32_t head = 0, lo[kStg], hi[kStg];
            int m = 0, oldest = 0, lastj = -1;
            bool ok = true;
            const uint64_t pol = l2_policy_evict_first();
            Cursor ic;
            cur_start(ic, p, lt, nj, nk);
            while (ic.j < nj && ok) {
                if (ic.j != lastj) {
                    if (lastj >= 0) stamp(p, jslot(lastj, 6));
                    stamp(p, jslot(ic.j, 5));
                    lastj = ic.j;
                }
                const Seg &g = ic.g;
                const int rows = min(g.rps, ic.nr - ic.row0);
                const uint32_t part = (uint32_t)(rows * g.rb), bytes = part * (g.w2 ? 2u : 1u);
                const uint32_t before = head;
                const uint32_t off = ring_next(head, bytes, (uint32_t)sm.ring);
                // a stage that wraps to offset 0 skips the tail [before, ring): stages still
                // recorded there are older than any at the start and leave the FIFO first
                const bool wrapped = off == 0 && before + bytes > (uint32_t)sm.ring;
                // the bytes (and the barrier slot) are free once the consumers read the stages there
                while (oldest < m && (m - oldest >= kStg ||
                                      (lo[oldest % kStg] < off + bytes && off < hi[oldest % kStg]) ||
                                      (wrapped && lo[oldest % kStg] >= before))) {
                    if (!mbar_wait_s(&cons[oldest % kStg], (oldest / kStg) & 1, p.status, ms)) ok = false;
                    oldest++;
                    if (!ok) break;
                }
                if (!ok) break;
                lo[m % kStg] = off;
                hi[m % kStg] = off + bytes;
                uint64_t *fb = &full[m % kStg];
                mbar_arrive_expect_tx(fb, bytes);
                const long long src = (long long)(ic.r0 + ic.row0) * g.rb;
                bulk_g2s_hint(ring + off, g.w + src, part, fb, pol);
                if (g.w2) bulk_g2s_hint(ring + off + part, g.w2 + src, part, fb, pol);
                m++;
                cur_step(ic, p, lt, nj, nk);
            }
            if (lastj >= 0) stamp(p, jslot(lastj, 6));
            // copies still in flight land before the block exits
            for (int u = max(0, m - kStg); u < m; u++) mbar_wait_s(&full[u % kStg], (u / kStg) & 1, p.status, ms);
            role_done(p, ms, ep);
        }
        return;
    }

    if (warp > kCW) {
        // ------------------------------------------------ chain warps
        const int c = warp - kCW - 1;
        int m = 0;
        bool failed = false;
        unsigned long long best = 0;  // greedy key of this lane's logits
        uint8_t *bad = smem + sm.off_bad;
        const uint32_t rec_s = smem_u32(smem + sm.off_rec);
        const int64_t pos = __ldcg(p.pos);
        if (c == 0)  // cos / sin of this position, for every RoPE of the step
            for (int i = lane; i < p.rotary / 2; i += 32) ms.rope[i] = __ldg(p.rope_cs + (size_t)pos * (p.rotary / 2) + i);
        bar_chain();
        for (int j = 0; j < nj; j++) {
            const int kind = j == 4 * p.L ? J_HEAD : j & 3, l = j >> 2;
            const StepLayer *ly = kind == J_HEAD ? nullptr : &lt[l];
            for (int s = 0; s < nsegs(kind); s++) {
                const Seg g = get_seg(p, lt, j, s, nk);
                if (g.kv) continue;  // attention stages: no records
                int r0, nr;
                seg_rows(g, cta, G, r0, nr);
                const int nb = g.nb, rstride = (nb + 1) * 16;
                for (int lo = 0; lo < nr; lo += g.rps, m++) {
                    if (m % kNC != c) continue;
                    const int rs = m % kRS;
                    if (!failed && !mbar_wait_s(&rdone[rs], (m / kRS) & 1, p.status, ms)) failed = true;
                    failed = __any_sync(FULLM, failed);
                    const int rows = min(g.rps, nr - lo), srows = g.w2 ? 2 * rows : rows;
                    for (int t0 = 0; t0 < srows; t0 += 32) {
                        const int sr = t0 + lane;           // stage row
                        const bool valid = sr < srows;
                        const int idx = rs * kRowsCap + (valid ? sr : 0);
                        const uint32_t rr = rec_s + (uint32_t)(rs * kRecStage + (valid ? sr : 0) * rstride);
                        // the matrix row: gate rows first, then the up rows of a paired stage
                        const bool upper = g.w2 && sr >= rows;
                        const int orow = r0 + lo + (upper ? sr - rows : sr);
                        // the residual row, fetched before the chain so its latency overlaps it
                        const float xres = ((kind == J_O || kind == J_DOWN) && valid) ? __ldcg(p.x + orow) : 0.f;
                        float tot = 0.f, off = 0.f;
                        if (valid) {
                            if (g.dt == Q4_K) {
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
                        const bool refused = valid && bad[idx] != 0;
                        if (valid) bad[idx] = 0;
                        float val = __fsub_rn(tot, off);
                        // refused rows: the f32 product of the row with the f32 activation
                        unsigned rm = __ballot_sync(FULLM, refused && !failed);
                        while (rm) {
                            const int i = __ffs(rm) - 1;
                            rm &= rm - 1;
                            const int sri = t0 + i;
                            const bool up_i = g.w2 && sri >= rows;
                            const int fr = r0 + lo + (up_i ? sri - rows : sri);
                            const uint8_t *wrow = (up_i ? g.w2 : g.w) + (long long)fr * g.rb;
                            float r;
                            if (kind == J_O) {
                                r = row_dot_f32_fn(g.dt, wrow, nb, [&](int e) { return __ldcg(p.att + e); });
                            } else if (kind == J_DOWN) {
                                r = row_dot_f32_fn(g.dt, wrow, nb, [&](int e) { return __ldcg(p.a + e); });
                            } else {
                                // normed activation, recomputed from the residual (unchanged until
                                // every chain of this product is done)
                                const float inv = ms.inv[kind == J_QKV ? 0 : kind == J_GU ? 1 : 2];
                                const float *wn = kind == J_QKV ? ly->attn_norm : kind == J_GU ? ly->ffn_norm
                                                                                                 : p.out_norm;
                                r = row_dot_f32_fn(g.dt, wrow, nb, [&](int e) {
                                    return __fmul_rn(__fmul_rn(__ldcg(p.x + e), inv), __ldg(wn + e));
                                });
                            }
                            if (lane == i) val = r;
                        }
                        // ---- epilogues
                        if (kind == J_QKV) {
                            // RoPE on adjacent pairs (fast.go:507-557, interleaved), then q to qh, k / v
                            // to the f16 cache at the token's position (prim.go:76-96, 278)
                            const int dd = orow % p.D, head = orow / p.D;
                            const float other = __shfl_xor_sync(FULLM, val, 1);
                            float out = val;
                            if (s < 2 && dd < p.rotary) {
                                const float2 cs = ms.rope[dd >> 1];
                                const float x1 = (dd & 1) ? other : val, x2 = (dd & 1) ? val : other;
                                out = (dd & 1) ? __fadd_rn(__fmul_rn(x2, cs.x), __fmul_rn(x1, cs.y))
                                               : __fsub_rn(__fmul_rn(x1, cs.x), __fmul_rn(x2, cs.y));
                            }
                            if (valid && !failed) {
                                if (s == 0) {
                                    __stcg(p.qh + orow, out);
                                } else {
                                    unsigned short *cache = (unsigned short *)(s == 1 ? ly->kc : ly->vc);
                                    __stcg(cache + ((size_t)head * p.C + pos) * p.D + dd,
                                           (unsigned short)f32_to_f16(out));
                                }
                            }
                        } else if (kind == J_O || kind == J_DOWN) {
                            if (valid && !failed) __stcg(p.x + orow, __fadd_rn(xres, val));
                        } else if (kind == J_GU) {
                            // SiLU(gate) * up (attn.go:59-73: the amd64 kernel below F & ~7, float64 above)
                            const float up = __shfl_down_sync(FULLM, val, rows & 31);
                            if (valid && !upper && !failed) {
                                const float y = orow < (p.F & ~7) ? silu_mul_amd64(val, up) : silu_mul_f64(val, up);
                                __stcg(p.a + orow, y);
                            }
                        } else {
                            if (valid && !failed) {
                                __stcg(p.logits + orow, val);
                                if (val == val) best = max(best, argmax_key(val, orow));
                                if (orow == 0 && val != val) best = ~0ull;  // a NaN first logit: index 0 wins
                            }
                        }
                    }
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(&rfree[rs]);
                        stage_stamp(p, m, 3);
                    }
                }
            }
            // ---- end of the job: both chain warps are done with this CTA's rows
            bar_chain();
            if (c == 0 && lane == 0) stamp(p, jslot(j, 4));
            if (kind == J_HEAD) {
                if (p.amax) {
                    for (int o = 16; o; o >>= 1) best = max(best, __shfl_xor_sync(FULLM, best, o));
                    if (lane == 0 && best && !failed) atomicMax(p.amax, best);
                }
            } else if (kind == J_GU) {
                // this CTA's gate rows by 256-element block of the SwiGLU output: the
                // CTA whose rows complete a block quantizes it for the down product
                // (the two chain warps take alternate completed blocks)
                const Seg g = get_seg(p, lt, j, 0, nk);
                int r0, nr;
                seg_rows(g, cta, G, r0, nr);
                const int b0 = r0 / 256, nbk = nr > 0 ? (r0 + nr - 1) / 256 - b0 + 1 : 0;
                if (c == 0) {
                    bool last = false;
                    if (lane < nbk) {
                        const int b = b0 + lane;
                        const int rin = min(r0 + nr, 256 * (b + 1)) - max(r0, 256 * b);
                        last = atom_acqrel(&blkctr[l * nfb + b], (unsigned)rin) + (unsigned)rin == 256u * (ep + 1);
                    }
                    const unsigned mask = __ballot_sync(FULLM, last);
                    if (lane == 0) ms.qmask = mask;
                }
                bar_chain();
                unsigned mask = ms.qmask, done = 0;
                for (int k = 0; mask; k++) {
                    const int bit = __ffs(mask) - 1;
                    mask &= mask - 1;
                    if (k % kNC != c) continue;
                    const int b = b0 + bit;
                    const float4 *src = (const float4 *)(p.a + b * 256 + 8 * lane);
                    const float4 v0 = __ldcg(src), v1 = __ldcg(src + 1);
                    const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
                    int qq[8], s16, s32;
                    float dx;
                    bool ok;
                    warp_quant(v, qq, s16, s32, dx, ok);
                    quant_store_global(p.actF, b, qq, s16, s32, dx, ok);
                    done++;
                }
                __syncwarp();
                if (lane == 0 && done) red_rel(&ctr[1 + 5 * l + C_QUANT], done);
            } else if (c == 0 && lane == 0) {
                red_rel(&ctr[1 + 5 * l + (kind == J_QKV ? C_QKV : kind == J_O ? C_O : C_DOWN)], 1u);
            }
        }
        if (lane == 0) role_done(p, ms, ep);
        return;
    }

    {
        // ---------------------------------------------------- consumers
        const uint32_t act_s = smem_u32(smem + sm.off_act), hdr_s = smem_u32(smem + sm.off_hdr);
        const uint32_t ys_s = smem_u32(smem + sm.off_ys), ring_s = smem_u32(ring);
        const uint32_t rec_s = smem_u32(smem + sm.off_rec);
        uint8_t *bad = smem + sm.off_bad;
        const int h = lane & 1;
        const int HU = attn_hu(p), units = p.H / HU;
        uint32_t head = 0;
        int m = 0, mr = 0;  // data stages (ring) and record stages consumed
        bool failed = false;
        if (threadIdx.x == 0) stamp(p, 0);
        // the token's embedding row (fast.go:818-842): this CTA's slice of x
        {
            const int32_t id = __ldcg(p.tok);
            int e0, ne;
            slab(p.E, cta, G, 1, e0, ne);
            const long long erb = row_bytes(p.embd_dt, p.E);
            for (int i = threadIdx.x; i < ne; i += kCT) {
                const float v = (id >= 0 && id < p.V) ? decode_elem(p.embd_dt, p.embd + id * erb, e0 + i) : 0.f;
                __stcg(p.x + e0 + i, v);
            }
            bar_cons();
            if (threadIdx.x == 0) red_rel(&ctr[0], 1u);
        }
        for (int j = 0; j < nj; j++) {
            const int kind = j == 4 * p.L ? J_HEAD : j & 3, l = j >> 2;
            // ---- the activation of this product into shared memory
            if (kind == J_QKV || kind == J_GU || kind == J_HEAD) {
                const unsigned *w = kind == J_QKV ? (l == 0 ? &ctr[0] : &ctr[1 + 5 * (l - 1) + C_DOWN])
                                    : kind == J_GU ? &ctr[1 + 5 * l + C_O]
                                                   : &ctr[1 + 5 * (p.L - 1) + C_DOWN];
                const float *wn = kind == J_QKV ? lt[l].attn_norm : kind == J_GU ? lt[l].ffn_norm : p.out_norm;
                norm_phase(p, wn, smem, sm, ms, kind == J_QKV ? 0 : kind == J_GU ? 1 : 2, w, (unsigned)G * (ep + 1),
                           jslot(j, 0));
            } else if (kind == J_O) {
                // attention units on the first CTAs, once every q / k / v row is written
                if (cta < units) {
                    if (threadIdx.x == 0) {
                        grid_wait(&ctr[1 + 5 * l + C_QKV], (unsigned)G * (ep + 1), p.status, ms);
                        stamp(p, jslot(j, 8));
                    }
                    bar_cons();
                    attn_unit(p, l, cta, HU, nk, smem, sm, ms, ring, full, cons, m, head, j);
                    bar_cons();
                    if (threadIdx.x == 0) {
                        red_rel(&ctr[1 + 5 * l + C_ATT], 1u);
                        stamp(p, jslot(j, 3));
                    }
                }
                if (threadIdx.x == 0) {
                    grid_wait(&ctr[1 + 5 * l + C_ATT], (unsigned)units * (ep + 1), p.status, ms);
                    stamp(p, jslot(j, 0));
                }
                bar_cons();
                stage_phase(p.actE, p.E, smem, sm, ms);
            } else {
                if (threadIdx.x == 0) {
                    grid_wait(&ctr[1 + 5 * l + C_QUANT], (unsigned)nfb * (ep + 1), p.status, ms);
                    stamp(p, jslot(j, 0));
                }
                bar_cons();
                stage_phase(p.actF, p.F, smem, sm, ms);
            }
            const bool act_ok = ms.act_ok != 0;
            if (threadIdx.x == 0) stamp(p, jslot(j, 1));
            // ---- the product's stages
            for (int s = 0; s < nsegs(kind); s++) {
                const Seg g = get_seg(p, lt, j, s, nk);
                if (g.kv) continue;  // the attention unit read its stages already
                int r0, nr;
                seg_rows(g, cta, G, r0, nr);
                const int nb = g.nb, sbk = (g.w2 ? 2 : 1) * g.rps * nb;
                const int dt = g.dt, bb = g.bb, rstride = (nb + 1) * 16;
                const int blk = dt == Q4_K ? 16 * warp + (lane >> 1) : 8 * (16 * (warp >> 3) + (lane >> 1)) + (warp & 7);
                const bool lane_on = blk < sbk;
                const int roff = blk / nb, kb = blk - roff * nb;
                const uint32_t ya = act_s + (uint32_t)act_off(lane_on ? kb : 0, h);
                const uint32_t ha = (uint32_t)hdr_off(2 * (lane_on ? kb : 0) + h);
                for (int row0 = 0; row0 < nr; row0 += g.rps, m++, mr++) {
                    const int rows = min(g.rps, nr - row0), srows = g.w2 ? 2 * rows : rows;
                    const uint32_t off = ring_next(head, (uint32_t)(srows * g.rb), (uint32_t)sm.ring);
                    const int slot = m % kStg, rs = mr % kRS;
                    if (!failed && !mbar_wait_s(&full[slot], (m / kStg) & 1, p.status, ms)) failed = true;
                    if (threadIdx.x == 0) stage_stamp(p, mr, 0);
                    if (!failed && mr >= kRS && !mbar_wait_s(&rfree[rs], ((mr / kRS) & 1) ^ 1, p.status, ms))
                        failed = true;
                    if (threadIdx.x == 0) stage_stamp(p, mr, 1);
                    failed = __any_sync(FULLM, failed);
                    const bool active = !failed && lane_on && roff < srows;
                    int S = 0, M = 0;
                    uint32_t dh = 0, mh = 0;
                    float dx = 0.f;
                    if (active) {
                        const uint32_t ba = ring_s + off + (uint32_t)(blk * bb);
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
                    S += __shfl_xor_sync(FULLM, S, 1);
                    M += __shfl_xor_sync(FULLM, M, 1);
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&cons[slot]);  // the stage's bytes go back to the producer
                    if (active && h == 0) {
                        const float d = f16f(dh);
                        float fm = 0.f, pm = 0.f;
                        bool nf = !f16_finite(dh) || !act_ok;
                        if (dt == Q4_K) {
                            fm = __int2float_rn(M);
                            pm = __fmul_rn(f16f(mh), dx);
                            nf |= !f16_finite(mh);
                        }
                        sts128(rec_s + (uint32_t)(rs * kRecStage + roff * rstride + kb * 16),
                               __float_as_uint(__int2float_rn(S)), __float_as_uint(__fmul_rn(d, dx)),
                               __float_as_uint(fm), __float_as_uint(pm));
                        if (nf) bad[rs * kRowsCap + roff] = 1;
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&rdone[rs]);
                    if (threadIdx.x == 0) stage_stamp(p, mr, 2);
                }
            }
            if (threadIdx.x == 0) stamp(p, jslot(j, 2));
        }
        __syncwarp();
        if (threadIdx.x == 0) stamp(p, 1);
        if (lane == 0) role_done(p, ms, ep);
    }
}

__global__ void rope_table_kernel(const double *inv_freq, int C, int half, float2 *cs) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= (long long)C * half) return;
    const int pos = (int)(i / half), k = (int)(i % half);
    double sd, cd;
    sincos(__dmul_rn((double)pos, inv_freq[k]), &sd, &cd);  // as rope_scatter_kernel
    cs[i] = make_float2((float)cd, (float)sd);
}

int act_region(int nbmax) {
    const int a = (act_bytes(nbmax) + 15) & ~15;
    return a + 2 * hdr_bytes(nbmax);
}

}  // namespace

bool step_ok(int E, int F, int H, int Hkv, int D, int C, int rotary, int interleaved, int cache_f16) {
    if (E % 256 || F % 256 || E < 2048 || F < 2048 || E > kMaxE || F > kMaxK) return false;
    if (D != 128 || Hkv <= 0 || H % Hkv || H * D != E || !interleaved || !cache_f16 || rotary % 2 || rotary > D)
        return false;
    const int G = H / Hkv, HU = 2;  // attention units of two query heads (one 256-element block)
    if (G % 2) return false;
    // attention scratch in the act + record regions: q, outputs and HU x C scores
    const int nbmax = (E > F ? E : F) / 256;
    const long long scratch = (long long)act_region(nbmax) + kRS * kRecStage;
    return (long long)attn_scratch_bytes(HU, C) <= scratch;
}

size_t step_sync_words(int L, int F) { return 1 + 5 * (size_t)L + (size_t)L * (F / 256); }

cudaError_t step_prepare() {
    static std::atomic<unsigned long long> done{0};
    return once_per_device(done, [] {
        return cudaFuncSetAttribute(step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    });
}

cudaError_t launch_step(const StepParams &p, cudaStream_t st) {
    cudaError_t e = step_prepare();
    if (e != cudaSuccess) return e;
    Smem sm;
    const int nbmax = (p.E > p.F ? p.E : p.F) / 256;
    sm.off_lt = (kMiscOff + (int)sizeof(Misc) + 15) & ~15;
    sm.off_act = (sm.off_lt + p.L * (int)sizeof(StepLayer) + 127) & ~127;
    sm.off_hdr = sm.off_act + ((act_bytes(nbmax) + 15) & ~15);
    sm.off_ys = sm.off_hdr + hdr_bytes(nbmax);
    sm.off_rec = (sm.off_ys + hdr_bytes(nbmax) + 127) & ~127;
    sm.off_bad = sm.off_rec + kRS * kRecStage;
    sm.off_ring = (sm.off_bad + kRS * kRowsCap + 127) & ~127;
    sm.ring = (kSmem - sm.off_ring) & ~127;
    if (sm.ring < 2 * 53760) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(num_sms());
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once: the grid counters need it
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, step_kernel, p, sm);
}

cudaError_t launch_rope_table(const double *inv_freq, int C, int half, float2 *cs, cudaStream_t st) {
    const long long n = (long long)C * half;
    if (n <= 0) return cudaSuccess;
    rope_table_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(inv_freq, C, half, cs);
    return cudaGetLastError();
}

}  // namespace mimgpu
