// kernels.h -- host-side launchers of the sm_100a kernels (internal API of
// libmimgpu; the public C ABI is include/mimgpu.h).
#pragma once

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace mimgpu {

// Runs `set` (kernel attributes, which are per device) once for the current
// device; `done` holds one bit per device ordinal and may be shared by
// threads and contexts.
template <class F>
cudaError_t once_per_device(std::atomic<unsigned long long> &done, F set) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const unsigned long long bit = 1ull << (dev & 63);
    if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
    e = set();
    if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_acq_rel);
    return e;
}

// 8-bit activations in blocks of 256 (internal/kernels/q8.go:50-97):
// q [rows,K] int8, dx [rows,K/256] scale amax/127, xs [rows,K/32] sums of
// each run of 32 quants, ys [rows,K/16] sums of each run of 16, and
// ok [rows,K/256] per block (0 when the block holds NaN, Inf or |x| > 2^60;
// the reference then refuses the whole row).
struct ActQ8 {
    int8_t *q;
    float *dx;
    int16_t *xs;
    int16_t *ys;
    int *ok;
};
size_t act_q8_bytes(int rows, long long K);
ActQ8 act_q8_carve(void *base, int rows, long long K);

// One weight matrix of a fused GEMV launch: W [n, K] in its block dtype,
// byte-exact rows of row_bytes(dt, K); y[a*ldy + j] for activation row a.
struct GemvSeg {
    const uint8_t *w;
    int dt;
    int n;
    float *y;
    long long ldy;
    const float *bias;  // [n] or null
    const float *res;   // residual added after the product (res[a*ldy + j]), or null
};

constexpr int kMaxSegs = 4;

// Room for the records of a split launch: a launch of 16-32 activation rows
// whose matrices have too few 128-row tiles to fill the SMs splits K over
// several CTAs, which store their exact block sums (8 bytes per weight row,
// activation row and block) for a second kernel that runs each pair's
// block-ordered chain.  Without it (or when it is too small) the launch is
// not split.  Same results bit for bit either way.
struct GemmSplit {
    int2 *rec;
    size_t bytes;
};

// One exchange of a tensor-parallel step through peer memory (p2p.cuh):
// N = 0 or 1 means none.  The producer stores into every rank's copy of a
// buffer at arena offset `off` (+ column `col0`); the consumer publishes
// this rank's part of slot `slot` and waits for every rank's.
struct P2P {
    const uint64_t *base;   // [N] arena base of every rank (device array; own included)
    long long off_flags;    // byte offset of the flag array [slots][N] (u32) in the arena
    const unsigned *epoch;  // this rank's forward counter
    unsigned *status;       // device status word
    int N, k, slot;
    long long off;          // producer: arena offset of the destination buffer
    long long col0;         // producer: first element of this rank's slice in it
};

// wait: an exchange the input depends on (consumer side), or null
cudaError_t launch_quantize_a8(const float *x, int rows, long long K, ActQ8 act, cudaStream_t st, bool pdl,
                               const P2P *wait = nullptr);
// y = rms_norm(x) * scale, and its 8-bit blocks (fast.go:434-485 then q8.go:50-97);
// act may have a null q (no quantization)
cudaError_t launch_rmsnorm_quant(const float *x, int rows, int n, const float *scale, float eps, float *y,
                                 ActQ8 act, cudaStream_t st, bool pdl, const P2P *wait = nullptr);
// y = silu(gate)*up (attn.go:63-73, float64) and its 8-bit blocks; act.q may be null
// put: store the (one-row) result into every rank's copy of the exchanged
// buffer and publish (producer side), or null
cudaError_t launch_swiglu_quant(const float *gate, const float *up, long long ldg, int rows, int n, float *y,
                                ActQ8 act, cudaStream_t st, bool pdl, const P2P *put = nullptr);
// dequant_matmul_a8.v2 block 256 over up to kMaxSegs Q4_K/Q6_K matrices
// sharing the activations.  x is the f32 input, used for refused rows.
// Sets the kernel attributes the GEMV launches need (call outside stream capture).
cudaError_t gemv_a8_prepare();
// cache_maps: keep each weight's TMA descriptor in a host table (false:
// encode it on the stack every launch, allocating nothing).
// put: the (one-segment, one-row) outputs also go to every rank's copy of
// the exchanged buffer, then the launch publishes (producer side)
// The next one-row GEMVs of a decode step, whose weights a launch prefetches
// into L2 once its own copies are all issued: for each target launch, each
// CTA takes the first `bytes` of its slabs of that launch's matrices, the
// bytes the target's CTA of the same index streams first, so the target
// starts from L2 while HBM would otherwise idle (its predecessor's tail, the
// small kernels between).  Targets are the next launch and, optionally, the
// one after it (the o GEMV prefetches little of its own successor's bytes
// while the attention runs unless the q|k|v GEMV before it starts early).
struct GemvPrefetchTarget {
    const uint8_t *w[kMaxSegs];
    int n[kMaxSegs], dt[kMaxSegs];
    int nseg, unit;
    long long K;
    uint32_t bytes;  // per slab, a multiple of 16
};
constexpr int kMaxPrefetchTargets = 2;
struct GemvPrefetch {
    GemvPrefetchTarget t[kMaxPrefetchTargets];
    int nt;
    int G;  // slabs (the launches' CTAs: one per SM)
};
// Adds the launch of segs over K as a target of pf (bytes per slab); false,
// leaving pf unchanged, when that launch would not be a one-row (slab) GEMV.
bool gemv_prefetch_add(const GemvSeg *segs, int nseg, long long K, uint32_t bytes, GemvPrefetch &pf);
// rms_norm of the row nrm.x fused into a one-row GEMV: every CTA makes its
// own 8-bit activations instead of reading act (CTA 0 also writes the
// normalised row to nrm.h, which must be the launch's x); same bits as
// launch_rmsnorm_quant followed by the GEMV.  Only where gemv_row_ok holds
// and K <= 8192.
struct GemvNorm {
    const float *x;      // [K] the residual row
    const float *scale;  // [K] or null
    float eps;
    float *h;            // [K] the normalised row
};
cudaError_t launch_gemv_a8(const GemvSeg *segs, int nseg, const float *x, ActQ8 act, int rows, long long K,
                           unsigned *status, cudaStream_t st, bool pdl, bool cache_maps = true,
                           const P2P *put = nullptr, const GemvPrefetch *pf = nullptr,
                           const GemvNorm *nrm = nullptr, const GemmSplit *split = nullptr);
// The same product on the tensor cores (tcgen05 kind::i8) for launches of
// at least kTcMinRows activation rows; launch_gemv_a8 dispatches to it.
constexpr int kTcMinRows = 16;
bool gemm_a8_tc_ok(const GemvSeg *segs, int nseg, const ActQ8 &act, int rows, long long K);
cudaError_t gemm_a8_tc_prepare();
// Bytes of records a launch of these matrices would split into (0: it would not split).
size_t gemm_a8_split_bytes(const GemvSeg *segs, int nseg, int rows, long long K);
cudaError_t launch_gemm_a8_tc(const GemvSeg *segs, int nseg, const float *x, ActQ8 act, int rows, long long K,
                              unsigned *status, cudaStream_t st, bool pdl, const GemmSplit *split = nullptr);
// The one-activation-row product (decode steps): one slab of consecutive
// rows per SM, streamed with bulk copies; launch_gemv_a8 dispatches to it
// when every matrix is a whole number of row units (the fewest rows whose
// bytes are a 16-byte multiple: 1 for Q4_K, 1, 2, 4 or 8 for Q6_K; see
// gemv_row_ok).  Same results bit for bit.
bool gemv_row_ok(const GemvSeg *segs, int nseg, const ActQ8 &act, long long K);
cudaError_t gemv_row_prepare();
cudaError_t launch_gemv_row(const GemvSeg *segs, int nseg, const float *x, ActQ8 act, long long K, unsigned *status,
                            cudaStream_t st, bool pdl, const P2P *put, const GemvPrefetch *pf = nullptr,
                            const GemvNorm *nrm = nullptr);
// dequant_matmul_a8.v1: 8-bit activations in blocks of 32 (q8.go:50-97) and
// the AVX2 block-32 row kernels restated bit for bit (k_a8_b32.cu).  The
// activation layout is ActQ8 with dx and xs per run of 32, ok per 256
// elements (the last one partial), ys unused.
size_t act_q8_b32_bytes(int rows, long long K);
ActQ8 act_q8_b32_carve(void *base, int rows, long long K);
// Q4_K and Q6_K with K % 256 == 0, Q8_0 with K % 32 == 0 (FusedQ8, q8.go:99-103)
bool a8_b32_dtype_ok(int dt, long long K);
cudaError_t launch_quantize_a8_b32(const float *x, int rows, long long K, ActQ8 act, cudaStream_t st);
cudaError_t launch_gemv_a8_b32(const GemvSeg &sg, const float *x, ActQ8 act, int rows, long long K, cudaStream_t st);
// dequant_matmul.v1: f32 activations, weights decoded exactly (Q4_K, Q6_K, Q8_0, F16, F32)
cudaError_t launch_gemv_f32(const GemvSeg *segs, int nseg, const float *x, int rows, long long K,
                            cudaStream_t st, bool pdl);

// dequantize n elements (quant.go Dequantize) and embedding rows (fast.go:818-842);
// the embedding launch of a step also advances the step counter `epoch` (may be null)
cudaError_t launch_dequantize(int dt, const uint8_t *src, float *dst, long long n, cudaStream_t st);
cudaError_t launch_embedding(int dt, const uint8_t *table, long long V, int E, const int32_t *ids, int n,
                             float *y, cudaStream_t st, bool pdl, unsigned *epoch = nullptr);

cudaError_t launch_rmsnorm(const float *x, int rows, int n, const float *scale, float eps, float *y,
                           cudaStream_t st, bool pdl);
// rope.v1 on x [B,H,T,D]; pos [pos_rows, T]; inv_freq [rotary/2] (float64)
cudaError_t launch_rope(const float *x, int B, int H, int T, int D, const int64_t *pos, int pos_rows,
                        const double *inv_freq, int rotary, int interleaved, float *y, cudaStream_t st,
                        bool pdl);
cudaError_t launch_swiglu(const float *a, const float *b, long long n, float *y, cudaStream_t st, bool pdl);
cudaError_t launch_add(const float *a, const float *b, long long n, float *y, cudaStream_t st, bool pdl);
cudaError_t launch_cast_f16(const float *x, uint16_t *y, long long n, cudaStream_t st);
// general attention.v1/v2 (per-op path): q [B,Hq,Tq,D] f32, k/v [B,Hkv,Tk,D] f32 or f16,
// mask bool with broadcast strides (elements) or null
struct AttnArgs {
    const float *q;
    const void *k, *v;
    int kv_f16;
    int B, Hq, Tq, D, Hkv, Tk;
    const uint8_t *mask;
    long long mst[4];
    float scale;
    int causal;
    float *out;
};
cudaError_t launch_attention(const AttnArgs &a, cudaStream_t st);
// Greedy pick over v[0..n) holding global indices i0..: folds the block
// maxima into *key (zero before the call); the index is
// 0xFFFFFFFF - (key & 0xFFFFFFFF), or 0 for a zero key or the all-ones key
// that a NaN v[0] sets when this slice holds the first index.
cudaError_t launch_argmax(const float *v, long long n, long long i0, bool holds_first, unsigned long long *key,
                          cudaStream_t st, bool pdl, int rows = 1, long long ldv = 0);

// One thread waits (bounded by the context's limit, acquire at system
// scope) until *addr == value; a wait that runs out sets DEV_TIMEOUT.
cudaError_t launch_wait_value(const uint32_t *addr, uint32_t value, unsigned *status, cudaStream_t st);

// seeded synthetic weights (k_synth.cu)
// elements [first, first + nelems) of the seeded stream (first a multiple of the block)
cudaError_t launch_synth(int dt, uint64_t seed, long long nelems, float mean, float sigma, uint8_t *out,
                         cudaStream_t st, long long first = 0);

int num_sms();

}  // namespace mimgpu
