// model.cu -- the llama graph of importer/llama.go:317-547 (gsoultan/mimir-model)
// as a device-resident step: mimgpu_model / mimgpu_session of include/mimgpu.h.
//
// One Session.Run (interp/interp.go:409-526) of the graph becomes one
// enqueue of ~10 kernels per layer on the session's stream, chained with
// programmatic dependent launch so each GEMV streams its weights while the
// previous kernel finishes.  The T = 1 step is captured once as a CUDA
// graph (positions and token ids are read from device memory, so the same
// graph serves every step); greedy generation replays it with the argmax and
// the position update inside, so nothing crosses the bus between steps.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <cstdlib>
#include <string>
#include <vector>

#include "common.cuh"
#include "ctx.h"
#include "kernels.h"
#include "model_kernels.h"
#include "step.h"

using namespace mimgpu;

namespace {

struct LayerW {
    const mimgpu_tensor *attn_norm = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr;
    const mimgpu_tensor *ffn_norm = nullptr, *gate = nullptr, *up = nullptr, *down = nullptr;
    // the query/key/value biases of a Qwen 2 graph (importer/llama.go:470-478:
    // the optional third input of the products), all three or none
    const mimgpu_tensor *bq = nullptr, *bk = nullptr, *bv = nullptr;
};

}  // namespace

struct mimgpu_model {
    mimgpu_ctx *ctx = nullptr;
    mimgpu_llama_config c{};
    const mimgpu_tensor *embd = nullptr, *out_norm = nullptr, *out = nullptr;
    std::vector<LayerW> L;
    double *inv_freq = nullptr;  // device [rope_dims/2]
    mimgpu_tp *tp = nullptr;     // tensor-parallel group, or null for one GPU
};

struct mimgpu_session {
    mimgpu_model *m = nullptr;
    cudaStream_t st = nullptr;
    std::vector<void *> kc, vc;
    size_t cache_bytes = 0;
    float *scores = nullptr;  // score scratch of the many-row attention (prompt passes), or null
    GemmSplit split{};        // records of split tensor-core GEMMs (16-32-row runs), or none
    void *arena = nullptr;
    float *x = nullptr, *h = nullptr, *qkv = nullptr, *qh = nullptr, *att = nullptr, *gu = nullptr, *a = nullptr;
    float *logits = nullptr;
    // tensor parallelism: this rank's slices before the all-gathers, and the
    // all-gather landing buffer ([ranks][T][width])
    float *attl = nullptr, *al = nullptr, *xl = nullptr, *logl = nullptr, *gbuf = nullptr;
    // peer-memory exchanges of the one-token step (p2p.cuh): flags [slots][N],
    // last-arrival counters [slots], the ranks' argmax keys [N], the forward
    // counter, and the table of every rank's arena base (IPC-mapped)
    unsigned *flags = nullptr, *counters = nullptr, *epoch = nullptr;
    unsigned long long *keys = nullptr;
    uint64_t *peer_base = nullptr;
    std::vector<void *> opened;  // peers' arenas mapped with cudaIpcOpenMemHandle
    bool p2p = false;
    ActQ8 actE{}, actF{};
    int32_t *tok = nullptr, *ids = nullptr;
    int64_t *pos = nullptr;
    unsigned long long *amax = nullptr;  // argmax keys [max_tokens], zero between steps
    int *step = nullptr;
    cudaGraphExec_t g_step = nullptr;    // T=1 forward, logits of the row
    cudaGraphExec_t g_greedy = nullptr;  // T=1 forward + argmax + advance
    // batched decoding: `slots` sequences, one cache each; a batched run's row
    // sequences (device [max_tokens]); the sequence of single-sequence runs
    int slots = 1;
    int32_t *slot = nullptr;
    int slot0 = 0;
    bool batched = false;                // the run in flight uses `slot`
    cudaGraphExec_t g_batch = nullptr;   // batched greedy step of g_batch_rows rows
    int g_batch_rows = 0;
    // the one-kernel decode step (k_step.cu), when the model qualifies
    bool step_ok = false, use_step = false;
    // one-row decode GEMVs prefetch the first bytes of each SM's slab of the
    // next GEMV (prefetch_next) and of the one after it (prefetch_skip) into
    // L2, by the kind of that GEMV: 0 q|k|v, 1 o, 2 gate|up, 3 down, 4 head
    // (mimgpu_session_set_l2_prefetch / _for; 0 = off)
    uint32_t prefetch_next[5] = {160 * 1024, 160 * 1024, 160 * 1024, 160 * 1024, 160 * 1024};
    uint32_t prefetch_skip[5] = {0, 0, 0, 0, 0};
    // one-token steps on one GPU: each rms_norm runs inside the GEMV that
    // reads it (GemvNorm) instead of as a kernel of its own
    bool fuse_norm = true;
    int step_kernels = 0;  // kernel launches in one replay of the greedy one-token graph
    // per layer: the key cache's tensor map for the decode attention
    std::vector<CUtensorMap> kmap;
    bool kmap_ok = false;
    StepLayer *step_layers = nullptr;    // device [layers]
    float2 *rope_cs = nullptr;           // device [context][rope_dims / 2]
    unsigned *step_sync = nullptr;       // grid counters, then [2] steps completed / CTA exits
    unsigned long long *trace = nullptr; // caller's timeline buffer of the step kernel, or null
};

namespace {

// d0 rows (or, for a tensor-parallel rank, shard rows: its own rows only) of d1
int check_shape(mimgpu_ctx *c, const char *name, const mimgpu_tensor *w, long long d0, long long d1,
                long long shard = -1) {
    if (!w) return fail(c, MIMGPU_EINVAL, "weight %s is missing", name);
    const bool rows_ok = w->shape[0] == d0 || (shard >= 0 && w->shape[0] == shard);
    const bool ok = d1 < 0 ? (w->ndim == 1 && w->shape[0] == d0) : (w->ndim == 2 && rows_ok && w->shape[1] == d1);
    if (!ok) return fail(c, MIMGPU_EINVAL, "weight %s has the wrong shape", name);
    return MIMGPU_OK;
}

bool matrix_dtype(int dt, bool a8) { return dt == Q4_K || dt == Q6_K || (!a8 && (dt == Q8_0 || dt == F16 || dt == F32)); }

int validate(mimgpu_model *m) {
    const auto &c = m->c;
    mimgpu_ctx *x = m->ctx;
    const int N = tp_size(m->tp), k = tp_rank(m->tp);
    if (N > 1 && (c.ffn % N || c.heads % N || c.kv_heads % N))
        return fail(x, MIMGPU_ENOTHANDLED,
                    "tensor parallelism over %d ranks needs ffn %d, heads %d and kv heads %d divisible by it", N, c.ffn,
                    c.heads, c.kv_heads);
    const long long E = c.embed, F = c.ffn, V = c.vocab, KV = (long long)c.kv_heads * c.head_dim;
    // a rank may hold only its rows of each matrix (the embedding table is read by token, whole)
    const long long sE = N > 1 ? E / N : -1, sF = N > 1 ? F / N : -1, sKV = N > 1 ? KV / N : -1;
    const long long Vl = (V + N - 1) / N, sV = N > 1 ? std::max(0LL, std::min(Vl, V - k * Vl)) : -1;
    int rc;
    if ((rc = check_shape(x, "token_embd.weight", m->embd, V, E))) return rc;
    if ((rc = check_shape(x, "output_norm.weight", m->out_norm, E, -1))) return rc;
    if (m->out && (rc = check_shape(x, "output.weight", m->out, V, E, sV))) return rc;
    if (m->out_norm->dtype != F32) return fail(x, MIMGPU_ENOTHANDLED, "norm weights must be f32");
    for (int l = 0; l < c.layers; l++) {
        const LayerW &w = m->L[l];
        const struct { const char *n; const mimgpu_tensor *t; long long d0, d1, shard; } list[] = {
            {"attn_norm", w.attn_norm, E, -1, -1}, {"attn_q", w.q, E, E, sE},      {"attn_k", w.k, KV, E, sKV},
            {"attn_v", w.v, KV, E, sKV},          {"attn_output", w.o, E, E, sE}, {"ffn_norm", w.ffn_norm, E, -1, -1},
            {"ffn_gate", w.gate, F, E, sF},       {"ffn_up", w.up, F, E, sF},     {"ffn_down", w.down, E, F, sE}};
        for (auto &e : list) {
            std::string n = "blk." + std::to_string(l) + "." + e.n + ".weight";
            if ((rc = check_shape(x, n.c_str(), e.t, e.d0, e.d1, e.shard))) return rc;
            if (e.d1 < 0 && e.t->dtype != F32) return fail(x, MIMGPU_ENOTHANDLED, "%s must be f32", n.c_str());
            if (e.d1 >= 0 && !matrix_dtype(e.t->dtype, c.a8))
                return fail(x, MIMGPU_ENOTHANDLED, "%s: dtype %d is not served", n.c_str(), e.t->dtype);
        }
        // biases: all three or none, f32 vectors of the matrix's rows (or this rank's)
        const bool any = w.bq || w.bk || w.bv;
        if (any && !(w.bq && w.bk && w.bv))
            return fail(x, MIMGPU_EINVAL, "blk.%d: attn_q/k/v biases come together", l);
        const struct { const char *n; const mimgpu_tensor *t; long long d0, shard; } bl[] = {
            {"attn_q", w.bq, E, sE}, {"attn_k", w.bk, KV, sKV}, {"attn_v", w.bv, KV, sKV}};
        for (auto &e : bl) {
            if (!any) break;
            const bool ok = e.t->dtype == F32 && e.t->ndim == 1 &&
                            (e.t->shape[0] == e.d0 || (e.shard >= 0 && e.t->shape[0] == e.shard));
            if (!ok) return fail(x, MIMGPU_EINVAL, "blk.%d.%s.bias must be f32 [%lld]", l, e.n, e.d0);
        }
    }
    const mimgpu_tensor *head = m->out ? m->out : m->embd;
    if (!matrix_dtype(head->dtype, c.a8)) return fail(x, MIMGPU_ENOTHANDLED, "output head dtype %d", head->dtype);
    return MIMGPU_OK;
}

// Rows [r0, r0 + rows) of a weight matrix of `full` rows and row length K as
// a GEMV segment: `w` is the whole matrix, or exactly this rank's rows (a
// tensor-parallel shard, which starts at row r0 of the whole).
GemvSeg slice(const mimgpu_tensor *w, long long K, long long full, long long r0, int rows, float *y, long long ldy,
              const float *res, const mimgpu_tensor *bias = nullptr) {
    const uint8_t *base = w->shape[0] == full ? w->dev + r0 * row_bytes(w->dtype, K) : w->dev;
    const float *b = bias ? (const float *)bias->dev + (bias->shape[0] == full ? r0 : 0) : nullptr;
    GemvSeg g{base, w->dtype, rows, y, ldy, b, res};
    return g;
}

// Enqueues one run of the graph for T tokens whose ids and positions are
// already in s->tok / s->pos.  Logits of every row (all_rows) or of the
// last row go to s->logits; with greedy, the argmax and step update follow.
//
// Tensor parallelism over N ranks (rank k) splits every matrix by output
// rows, so each rank computes complete block-ordered dot products and the
// ranks' results are the one-GPU results bit for bit:
//   q|k|v    the rows of this rank's query heads [k H/N, (k+1) H/N) and kv
//            heads [k Hkv/N, (k+1) Hkv/N); RoPE, the key-value cache and
//            attention run on those heads only;
//   exchange the attention output (this rank's E/N columns to every rank);
//   o        output rows [k E/N, (k+1) E/N) over the whole attention output;
//   exchange the residual columns;
//   gate|up  rows [k F/N, (k+1) F/N); exchange the SwiGLU output;
//   down     output rows [k E/N, (k+1) E/N); exchange the residual columns;
//   head     vocabulary rows, then the greedy keys' maximum.
// Four exchanges per layer: NCCL all-gathers (prompt passes, or before the
// ranks' arenas are mapped) or peer-memory stores fused into the producing
// kernels (p2p.cuh).  No weight byte is read by two ranks (the norms and the
// one embedding row per token excepted).
cudaError_t enqueue_forward(mimgpu_session *s, int T, bool all_rows, bool greedy, unsigned *status) {
    mimgpu_model *m = s->m;
    const auto &c = m->c;
    const int E = c.embed, F = c.ffn, H = c.heads, Hkv = c.kv_heads, D = c.head_dim;
    const int N = tp_size(m->tp), k = tp_rank(m->tp);
    const int El = E / N, Fl = F / N, Hl = H / N, Hkvl = Hkv / N, KVl = Hkvl * D, KV = Hkv * D;
    const int Vl = (c.vocab + N - 1) / N, v0 = k * Vl, vn = std::max(0, std::min(Vl, c.vocab - v0));
    const long long ldq = El + 2LL * KVl;
    const bool a8 = c.a8 != 0;
    cudaStream_t st = s->st;
    const bool pdl = true;
    cudaError_t e;
#define CK(x)                              \
    do {                                   \
        if ((e = (x)) != cudaSuccess) return e; \
    } while (0)
    const ActQ8 none{};
    // peer-memory exchanges (the one-token step once the ranks' arenas are mapped)
    const bool p2p = N > 1 && T == 1 && s->p2p;
    auto aoff = [&](const void *ptr) { return (long long)((const uint8_t *)ptr - (const uint8_t *)s->arena); };
    auto xch = [&](int slot, const void *dst, long long col0) {
        P2P x{};
        x.base = s->peer_base;
        x.off_flags = aoff(s->flags);
        x.epoch = s->epoch;
        x.status = status;
        x.N = N;
        x.k = k;
        x.slot = slot;
        x.off = dst ? aoff(dst) : 0;
        x.col0 = col0;
        return x;
    };
    // all-gathers: this rank's [T][W] slab -> [T][N*W] in `full`
    auto gather = [&](const float *mine, int W, float *full) -> cudaError_t {
        if (T == 1) return tp_allgather(m->tp, mine, full, (size_t)W, st);
        cudaError_t r = tp_allgather(m->tp, mine, s->gbuf, (size_t)T * W, st);
        if (r == cudaSuccess) r = launch_unshard(s->gbuf, N, T, W, full, (long long)N * W, (long long)N * W, st);
        return r;
    };
    // the residual columns [k El, (k+1) El) this rank just wrote, to every rank (NCCL)
    auto gather_x = [&]() -> cudaError_t {
        if (T == 1) return tp_allgather(m->tp, s->x + (long long)k * El, s->x, (size_t)El, st);
        cudaError_t r = launch_pack(s->x, T, E, (long long)k * El, El, s->xl, st);
        if (r == cudaSuccess) r = gather(s->xl, El, s->x);
        return r;
    };
    // The GEMV launches of a forward in order -- per layer q|k|v, o, gate|up,
    // down, then the head -- as segments (weights and rows only), and the
    // L2 prefetch each one-token launch issues for the launch after it (the
    // head's is the next step's first q|k|v).
    const mimgpu_tensor *headt = m->out ? m->out : m->embd;
    auto segs_of = [&](int l, int which, GemvSeg *g) -> int {
        if (which == 4) {
            if (vn <= 0) return 0;
            g[0] = slice(headt, E, c.vocab, v0, vn, nullptr, 0, nullptr);
            return 1;
        }
        const LayerW &w = m->L[l];
        switch (which) {
        case 0:
            g[0] = slice(w.q, E, E, (long long)k * El, El, nullptr, 0, nullptr);
            g[1] = slice(w.k, E, KV, (long long)k * KVl, KVl, nullptr, 0, nullptr);
            g[2] = slice(w.v, E, KV, (long long)k * KVl, KVl, nullptr, 0, nullptr);
            return 3;
        case 1: g[0] = slice(w.o, E, E, (long long)k * El, El, nullptr, 0, nullptr); return 1;
        case 2:
            g[0] = slice(w.gate, E, F, (long long)k * Fl, Fl, nullptr, 0, nullptr);
            g[1] = slice(w.up, E, F, (long long)k * Fl, Fl, nullptr, 0, nullptr);
            return 2;
        default: g[0] = slice(w.down, F, E, (long long)k * El, El, nullptr, 0, nullptr); return 1;
        }
    };
    // the launch after (l, which): q|k|v, o, gate|up, down per layer, then
    // the head, then the next step's first q|k|v
    auto after = [&](int &l, int &which) {
        if (which == 3) {
            l++;
            which = l < c.layers ? 0 : 4;
        } else if (which == 4) {
            l = 0;
            which = 0;
        } else {
            which++;
        }
    };
    GemvPrefetch pfbuf;
    auto next_pf = [&](int l, int which) -> const GemvPrefetch * {
        if (T != 1 || !a8) return nullptr;
        pfbuf = GemvPrefetch{};
        int nl = l, nw = which;
        for (int d = 0; d < 2; d++) {
            after(nl, nw);
            const uint32_t bytes = d == 0 ? s->prefetch_next[nw] : s->prefetch_skip[nw];
            GemvSeg g[kMaxSegs];
            const int ns = bytes ? segs_of(nl, nw, g) : 0;
            if (ns > 0) gemv_prefetch_add(g, ns, nw == 3 ? F : E, bytes, pfbuf);
        }
        return pfbuf.nt ? &pfbuf : nullptr;
    };
    auto fuse_norm = [&](const GemvSeg *g, int n) {
        return s->fuse_norm && T == 1 && N == 1 && a8 && E <= 8192 && gemv_row_ok(g, n, s->actE, E);
    };
    CK(launch_embedding(m->embd->dtype, m->embd->dev, c.vocab, E, s->tok, T, s->x, st, pdl, s->epoch));
    for (int l = 0; l < c.layers; l++) {
        const LayerW &w = m->L[l];
        // exchange slots of the layer: 4l attention output, 4l+1 residual after o,
        // 4l+2 SwiGLU output, 4l+3 residual after down
        const P2P xin = xch(4 * (l - 1) + 3, nullptr, 0);
        GemvSeg qkv[3] = {slice(w.q, E, E, (long long)k * El, El, s->qkv, ldq, nullptr, w.bq),
                          slice(w.k, E, KV, (long long)k * KVl, KVl, s->qkv + El, ldq, nullptr, w.bk),
                          slice(w.v, E, KV, (long long)k * KVl, KVl, s->qkv + El + KVl, ldq, nullptr, w.bv)};
        const GemvNorm n_attn{s->x, (const float *)w.attn_norm->dev, (float)c.norm_eps, s->h};
        const bool f_attn = fuse_norm(qkv, 3);
        if (!f_attn)
            CK(launch_rmsnorm_quant(s->x, T, E, (const float *)w.attn_norm->dev, (float)c.norm_eps, s->h,
                                    a8 ? s->actE : none, st, pdl, (p2p && l > 0) ? &xin : nullptr));
        if (a8)
            CK(launch_gemv_a8(qkv, 3, s->h, s->actE, T, E, status, st, pdl, true, nullptr, next_pf(l, 0),
                              f_attn ? &n_attn : nullptr, &s->split));
        else CK(launch_gemv_f32(qkv, 3, s->h, T, E, st, pdl));
        AttnArgs2 aa{s->qh, s->kc[l], s->vc[l], s->pos, T, Hl, Hkvl, D, c.context, c.cache_f16,
                     (float)(1.0 / std::sqrt((double)D)), N > 1 ? s->attl : s->att, none, status, s->scores,
                     s->batched ? s->slot : nullptr, s->slot0};
        // decode rows (one token per sequence): RoPE, the cache write and the
        // attention in one kernel; prompt passes: RoPE + scatter, then attention
        const bool fused = s->rope_cs && s->kmap_ok && attn_decode_ok(aa);
        auto attend = [&](const AttnArgs2 &x) -> cudaError_t {
            if (!fused) return launch_attn_exact(x, st, pdl);
            AttnDecodeArgs da{};
            da.kmap[0] = s->kmap[2 * l];
            da.kmap[1] = s->kmap[2 * l + 1];
            da.at = x;
            da.qkv = s->qkv;
            da.ldq = ldq;
            da.rope_cs = s->rope_cs;
            da.rotary = c.rope_dims;
            da.interleaved = c.interleaved;
            return launch_attn_decode(da, st, pdl);
        };
        if (!fused) {
            RopeScatterArgs ra{s->qkv, ldq, s->pos, m->inv_freq, T, Hl, Hkvl, D, c.context, c.rope_dims,
                               c.interleaved, c.cache_f16, s->qh, s->kc[l], s->vc[l],
                               s->batched ? s->slot : nullptr, s->slot0, s->rope_cs};
            CK(launch_rope_scatter(ra, st, pdl));
        }
        const P2P attx = xch(4 * l, s->att, (long long)k * El);
        if (N > 1) {
            if (p2p) aa.put = attx;  // the heads of this rank into every rank's attention output
            CK(attend(aa));
            if (!p2p) CK(gather(s->attl, El, s->att));
            if (a8) CK(launch_quantize_a8(s->att, T, E, s->actE, st, pdl, p2p ? &attx : nullptr));
        } else if (!fused && attn_prefill_ok(aa)) {
            // a prompt pass: the many-row kernel, then the 8-bit blocks of its output
            CK(launch_attn_exact(aa, st, pdl));
            if (a8) CK(launch_quantize_a8(s->att, T, E, s->actE, st, pdl));
        } else {
            if (a8) aa.act = s->actE;  // quantized inside the one-row kernel
            CK(attend(aa));
        }
        GemvSeg o = slice(w.o, E, E, (long long)k * El, El, s->x + (long long)k * El, E, s->x + (long long)k * El);
        const P2P oput = xch(4 * l + 1, s->x, (long long)k * El);
        if (a8)
            CK(launch_gemv_a8(&o, 1, s->att, s->actE, T, E, status, st, pdl, true, p2p ? &oput : nullptr,
                              next_pf(l, 1), nullptr, &s->split));
        else CK(launch_gemv_f32(&o, 1, s->att, T, E, st, pdl));
        if (N > 1 && !p2p) CK(gather_x());
        GemvSeg gu[2] = {slice(w.gate, E, F, (long long)k * Fl, Fl, s->gu, 2LL * Fl, nullptr),
                         slice(w.up, E, F, (long long)k * Fl, Fl, s->gu + Fl, 2LL * Fl, nullptr)};
        const GemvNorm n_ffn{s->x, (const float *)w.ffn_norm->dev, (float)c.norm_eps, s->h};
        const bool f_ffn = fuse_norm(gu, 2);
        if (!f_ffn)
            CK(launch_rmsnorm_quant(s->x, T, E, (const float *)w.ffn_norm->dev, (float)c.norm_eps, s->h,
                                    a8 ? s->actE : none, st, pdl, p2p ? &oput : nullptr));
        if (a8)
            CK(launch_gemv_a8(gu, 2, s->h, s->actE, T, E, status, st, pdl, true, nullptr, next_pf(l, 2),
                              f_ffn ? &n_ffn : nullptr, &s->split));
        else CK(launch_gemv_f32(gu, 2, s->h, T, E, st, pdl));
        const P2P aput = xch(4 * l + 2, s->a, (long long)k * Fl);
        CK(launch_swiglu_quant(s->gu, s->gu + Fl, 2LL * Fl, T, Fl, N > 1 ? s->al : s->a,
                               (a8 && N == 1) ? s->actF : none, st, pdl, p2p ? &aput : nullptr));
        if (N > 1) {
            if (!p2p) CK(gather(s->al, Fl, s->a));
            if (a8) CK(launch_quantize_a8(s->a, T, F, s->actF, st, pdl, p2p ? &aput : nullptr));
        }
        GemvSeg dn = slice(w.down, F, E, (long long)k * El, El, s->x + (long long)k * El, E, s->x + (long long)k * El);
        const P2P xput = xch(4 * l + 3, s->x, (long long)k * El);
        if (a8)
            CK(launch_gemv_a8(&dn, 1, s->a, s->actF, T, F, status, st, pdl, true, p2p ? &xput : nullptr,
                              next_pf(l, 3), nullptr, &s->split));
        else CK(launch_gemv_f32(&dn, 1, s->a, T, F, st, pdl));
        if (N > 1 && !p2p) CK(gather_x());
    }
    const int first = all_rows ? 0 : T - 1, rows = T - first;
    const P2P xlast = xch(4 * (c.layers - 1) + 3, nullptr, 0);
    const mimgpu_tensor *head = headt;
    // vocabulary rows [v0, v0 + vn); one GPU writes the logits directly (the
    // tied embedding, when it is the head, is bound whole on every rank)
    float *lg = N > 1 ? s->logl : s->logits;
    const long long ldl = N > 1 ? Vl : c.vocab;
    GemvSeg hs = slice(head, E, c.vocab, v0, vn > 0 ? vn : 0, lg, ldl, nullptr);
    const GemvNorm n_out{s->x, (const float *)m->out_norm->dev, (float)c.norm_eps, s->h};
    const bool f_out = vn > 0 && rows == 1 && fuse_norm(&hs, 1);
    if (!f_out)
        CK(launch_rmsnorm_quant(s->x + (long long)first * E, rows, E, (const float *)m->out_norm->dev,
                                (float)c.norm_eps, s->h, a8 ? s->actE : none, st, pdl, p2p ? &xlast : nullptr));
    if (vn > 0) {
        if (a8)
            CK(launch_gemv_a8(&hs, 1, s->h, s->actE, rows, E, status, st, pdl, true, nullptr, next_pf(0, 4),
                              f_out ? &n_out : nullptr, &s->split));
        else CK(launch_gemv_f32(&hs, 1, s->h, rows, E, st, pdl));
    }
    if (greedy) {
        const P2P kput = xch(4 * c.layers, s->keys, 0);
        CK(launch_argmax(lg, vn, v0, k == 0, s->amax, st, pdl, rows, ldl));
        if (N > 1 && !p2p) CK(tp_allreduce_max_u64(m->tp, s->amax, st, (size_t)rows));
        CK(launch_advance(s->amax, s->tok, s->pos, s->ids, s->step, st, pdl, p2p ? &kput : nullptr, s->keys,
                          rows));
    } else if (N > 1) {
        // the whole vocabulary on every rank: [N][rows][Vl] -> [rows][vocab]
        CK(tp_allgather(m->tp, s->logl, s->gbuf, (size_t)rows * Vl, st));
        CK(launch_unshard(s->gbuf, N, rows, Vl, s->logits, c.vocab, c.vocab, st));
    }
#undef CK
    return cudaSuccess;
}

// The T = 1 step of sequence 0 as one persistent kernel (k_step.cu); with
// greedy, the key folded by the head's chain warps becomes the next token.
cudaError_t enqueue_step(mimgpu_session *s, bool greedy, unsigned *status) {
    const mimgpu_model *m = s->m;
    const auto &c = m->c;
    const mimgpu_tensor *head = m->out ? m->out : m->embd;
    StepParams p{};
    p.layers = s->step_layers;
    p.L = c.layers;
    p.E = c.embed;
    p.F = c.ffn;
    p.H = c.heads;
    p.Hkv = c.kv_heads;
    p.D = c.head_dim;
    p.V = c.vocab;
    p.C = c.context;
    p.rotary = c.rope_dims;
    p.eps = (float)c.norm_eps;
    p.scale = (float)(1.0 / std::sqrt((double)c.head_dim));
    p.embd = m->embd->dev;
    p.embd_dt = m->embd->dtype;
    p.head = head->dev;
    p.head_dt = head->dtype;
    p.out_norm = (const float *)m->out_norm->dev;
    p.rope_cs = s->rope_cs;
    p.tok = s->tok;
    p.pos = s->pos;
    p.x = s->x;
    p.qh = s->qh;
    p.att = s->att;
    p.a = s->a;
    p.logits = s->logits;
    p.actE = s->actE;
    p.actF = s->actF;
    p.amax = greedy ? s->amax : nullptr;
    p.sync = s->step_sync;
    p.epoch = s->step_sync + step_sync_words(c.layers, c.ffn);
    p.status = status;
    p.trace = s->trace;
    cudaError_t e = launch_step(p, s->st);
    if (e == cudaSuccess && greedy) e = launch_advance(s->amax, s->tok, s->pos, s->ids, s->step, s->st, false);
    return e;
}

// rows > 1: a batched step (row r of sequence slot[r], logits of every row)
int capture(mimgpu_session *s, bool greedy, cudaGraphExec_t *out, int rows = 1) {
    mimgpu_ctx *c = s->m->ctx;
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamBeginCapture(s->st, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) return cuda_fail(c, e, "begin capture");
    s->batched = rows > 1;
    cudaError_t fe = (rows == 1 && s->use_step) ? enqueue_step(s, greedy, c->status)
                                                : enqueue_forward(s, rows, rows > 1, greedy, c->status);
    s->batched = false;
    e = cudaStreamEndCapture(s->st, &g);
    if (fe != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        return cuda_fail(c, fe, "capture forward");
    }
    if (e != cudaSuccess) return cuda_fail(c, e, "end capture");
    // the kernel launches one replay makes (reported by mimgpu_session_step_kernels)
    size_t nn = 0;
    int kernels = 0;
    if (cudaGraphGetNodes(g, nullptr, &nn) == cudaSuccess && nn) {
        std::vector<cudaGraphNode_t> nodes(nn);
        if (cudaGraphGetNodes(g, nodes.data(), &nn) == cudaSuccess)
            for (size_t i = 0; i < nn; i++) {
                cudaGraphNodeType t;
                if (cudaGraphNodeGetType(nodes[i], &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) kernels++;
            }
    }
    if (greedy && rows == 1) s->step_kernels = kernels;
    e = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    return cuda_fail(c, e, "instantiate");
}

// Device state of the one-kernel step for a single-GPU a8 model whose
// dimensions qualify (step_ok): the layer table, the RoPE cos/sin table and
// the grid counters (zero; they only ever grow).
int setup_step(mimgpu_session *s) {
    mimgpu_model *m = s->m;
    const auto &c = m->c;
    mimgpu_ctx *x = m->ctx;
    const mimgpu_tensor *head = m->out ? m->out : m->embd;
    bool ok = tp_size(m->tp) == 1 && c.a8 && (head->dtype == Q4_K || head->dtype == Q6_K) &&
              step_ok(c.embed, c.ffn, c.heads, c.kv_heads, c.head_dim, c.context, c.rope_dims, c.interleaved,
                      c.cache_f16);
    for (int l = 0; l < c.layers && ok; l++) {
        const LayerW &w = m->L[l];
        const mimgpu_tensor *mats[7] = {w.q, w.k, w.v, w.o, w.gate, w.up, w.down};
        for (auto *t : mats) ok &= t->dtype == Q4_K || t->dtype == Q6_K;
        ok &= !w.bq;  // the step kernel has no bias inputs
        ok &= w.gate->dtype == w.up->dtype;
    }
    if (!ok) return MIMGPU_OK;
    std::vector<StepLayer> host(c.layers);
    for (int l = 0; l < c.layers; l++) {
        const LayerW &w = m->L[l];
        const mimgpu_tensor *mats[7] = {w.q, w.k, w.v, w.o, w.gate, w.up, w.down};
        for (int i = 0; i < 7; i++) {
            host[l].w[i] = mats[i]->dev;
            host[l].dt[i] = mats[i]->dtype;
        }
        host[l].attn_norm = (const float *)w.attn_norm->dev;
        host[l].ffn_norm = (const float *)w.ffn_norm->dev;
        host[l].kc = s->kc[l];
        host[l].vc = s->vc[l];
    }
    const size_t words = step_sync_words(c.layers, c.ffn) + 2;
    const int half = c.rope_dims / 2;
    if (!s->rope_cs) return MIMGPU_OK;
    cudaError_t e = cudaMalloc(&s->step_layers, host.size() * sizeof(StepLayer));
    if (e == cudaSuccess) e = cudaMalloc(&s->step_sync, words * sizeof(unsigned));
    if (e == cudaSuccess)
        e = cudaMemcpy(s->step_layers, host.data(), host.size() * sizeof(StepLayer), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(s->step_sync, 0, words * sizeof(unsigned));
    if (e == cudaSuccess) e = step_prepare();
    if (e == cudaSuccess) e = cudaStreamSynchronize(s->st);
    if (e != cudaSuccess) return cuda_fail(x, e, "step kernel setup");
    // available, off by default: measured slower than the kernel-per-op path
    // (8B shape 2.45 vs 2.08 ms per token, 70B 13.0 vs 10.2 ms on one B200)
    s->step_ok = true;
    s->use_step = false;
    return MIMGPU_OK;
}

void free_session(mimgpu_session *s) {
    if (!s) return;
    cudaSetDevice(s->m->ctx->device);
    if (s->st) cudaStreamSynchronize(s->st);
    if (s->g_step) cudaGraphExecDestroy(s->g_step);
    if (s->g_greedy) cudaGraphExecDestroy(s->g_greedy);
    if (s->g_batch) cudaGraphExecDestroy(s->g_batch);
    if (s->step_layers) cudaFree(s->step_layers);
    if (s->rope_cs) cudaFree(s->rope_cs);
    if (s->step_sync) cudaFree(s->step_sync);
    for (void *p : s->kc) cudaFree(p);
    for (void *p : s->vc) cudaFree(p);
    for (void *p : s->opened) cudaIpcCloseMemHandle(p);
    if (s->arena) cudaFree(s->arena);
    if (s->scores) cudaFree(s->scores);
    if (s->split.rec) cudaFree(s->split.rec);
    if (s->st) cudaStreamDestroy(s->st);
    delete s;
}

}  // namespace

extern "C" {

int mimgpu_model_new(mimgpu_ctx *ctx, const mimgpu_llama_config *cfg, mimgpu_model **out) {
    if (!ctx || !cfg || !out) return MIMGPU_EINVAL;
    std::lock_guard<std::recursive_mutex> lk(ctx->mu);
    *out = nullptr;
    const auto &c = *cfg;
    if (c.layers <= 0 || c.embed <= 0 || c.ffn <= 0 || c.heads <= 0 || c.kv_heads <= 0 || c.heads % c.kv_heads ||
        c.head_dim <= 0 || c.heads * c.head_dim != c.embed || c.vocab <= 0 || c.context <= 0 || c.max_tokens <= 0 ||
        c.max_tokens > c.context)
        return fail(ctx, MIMGPU_EINVAL, "llama config is inconsistent");
    if (c.rope_dims <= 0 || c.rope_dims % 2 || c.rope_dims > c.head_dim)
        return fail(ctx, MIMGPU_EINVAL, "rope dimension count %d for head size %d", c.rope_dims, c.head_dim);
    if (c.head_dim % 32 || 256 % c.head_dim)
        return fail(ctx, MIMGPU_ENOTHANDLED, "head size %d not served (32, 64, 128 or 256)", c.head_dim);
    if (attn_exact_smem(c.heads, c.kv_heads, c.head_dim, c.context, c.cache_f16) > kAttnSmemMax)
        return fail(ctx, MIMGPU_ENOTHANDLED, "context %d too long for the attention scores in shared memory", c.context);
    if (c.a8 && (c.embed % 256 || c.ffn % 256))
        return fail(ctx, MIMGPU_ENOTHANDLED, "8-bit activations need E and F multiples of 256");
    int rc = use_device(ctx);
    if (rc) return rc;
    auto *m = new mimgpu_model;
    m->ctx = ctx;
    m->c = c;
    m->L.resize(c.layers);
    std::vector<double> inv(c.rope_dims / 2);
    for (int i = 0; i < c.rope_dims / 2; i++) inv[i] = std::pow(c.rope_theta, -2.0 * (double)i / (double)c.rope_dims);
    cudaError_t e = cudaMalloc(&m->inv_freq, inv.size() * sizeof(double));
    if (e == cudaSuccess) e = cudaMemcpy(m->inv_freq, inv.data(), inv.size() * sizeof(double), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        if (m->inv_freq) cudaFree(m->inv_freq);
        delete m;
        return cuda_fail(ctx, e, "model");
    }
    *out = m;
    return MIMGPU_OK;
}

int mimgpu_model_set_weight(mimgpu_model *m, const char *name, const mimgpu_tensor *w) {
    if (!m || !name || !w) return MIMGPU_EINVAL;
    if (w->ctx != m->ctx) return fail(m->ctx, MIMGPU_EINVAL, "weight %s belongs to another context", name);
    if (!strcmp(name, "token_embd.weight")) { m->embd = w; return MIMGPU_OK; }
    if (!strcmp(name, "output_norm.weight")) { m->out_norm = w; return MIMGPU_OK; }
    if (!strcmp(name, "output.weight")) { m->out = w; return MIMGPU_OK; }
    int l = -1, used = 0;
    char rest[64] = {0};
    if (sscanf(name, "blk.%d.%63s%n", &l, rest, &used) != 2 || l < 0 || l >= m->c.layers)
        return fail(m->ctx, MIMGPU_EINVAL, "unknown weight %s", name);
    LayerW &L = m->L[l];
    const struct { const char *n; const mimgpu_tensor **slot; } names[] = {
        {"attn_norm.weight", &L.attn_norm}, {"attn_q.weight", &L.q},       {"attn_k.weight", &L.k},
        {"attn_v.weight", &L.v},           {"attn_output.weight", &L.o},  {"ffn_norm.weight", &L.ffn_norm},
        {"ffn_gate.weight", &L.gate},      {"ffn_up.weight", &L.up},      {"ffn_down.weight", &L.down},
        {"attn_q.bias", &L.bq},            {"attn_k.bias", &L.bk},        {"attn_v.bias", &L.bv}};
    for (auto &e : names)
        if (!strcmp(rest, e.n)) {
            *e.slot = w;
            return MIMGPU_OK;
        }
    return fail(m->ctx, MIMGPU_EINVAL, "unknown weight %s", name);
}

int mimgpu_model_set_tp(mimgpu_model *m, mimgpu_tp *tp) {
    if (!m) return MIMGPU_EINVAL;
    m->tp = tp;
    return MIMGPU_OK;
}

void mimgpu_model_free(mimgpu_model *m) {
    if (!m) return;
    cudaSetDevice(m->ctx->device);
    if (m->inv_freq) cudaFree(m->inv_freq);
    delete m;
}

int mimgpu_session_new(mimgpu_model *m, mimgpu_session **out) { return mimgpu_session_new_slots(m, 1, out); }

int mimgpu_session_new_slots(mimgpu_model *m, int slots, mimgpu_session **out) {
    if (!m || !out) return MIMGPU_EINVAL;
    mimgpu_ctx *c = m->ctx;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    *out = nullptr;
    if (slots < 1 || slots > m->c.max_tokens || slots > 1024)
        return fail(c, MIMGPU_EINVAL, "%d sequences; a session holds 1..min(max_tokens, 1024)", slots);
    int rc = validate(m);
    if (rc || (rc = use_device(c))) return rc;
    if ((rc = cuda_fail(c, gemv_a8_prepare(), "gemv setup"))) return rc;
    const auto &k = m->c;
    auto *s = new mimgpu_session;
    s->m = m;
    const long long T = k.max_tokens, E = k.embed, F = k.ffn, V = k.vocab, H = k.heads, D = k.head_dim;
    const long long KV = (long long)k.kv_heads * D;
    const long long N = tp_size(m->tp), El = E / N, Fl = F / N, Vl = (V + N - 1) / N;
    const long long gw = std::max(std::max(El, Fl), Vl);
    auto al = [](size_t b) { return (b + 255) & ~(size_t)255; };
    auto tpb = [&](size_t b) { return N > 1 ? al(b) : (size_t)0; };
    size_t bytes = 0;
    const size_t sz[] = {al(T * E * 4), al(T * E * 4), al(T * (E + 2 * KV) * 4), al(T * E * 4), al(T * E * 4),
                         al(T * 2 * F * 4), al(T * F * 4), al(T * V * 4), act_q8_bytes((int)T, E), act_q8_bytes((int)T, F),
                         al(T * 4), al(T * 8), al(65536 * 4), al(256),
                         tpb(T * El * 4), tpb(T * Fl * 4), tpb(T * El * 4), tpb(T * Vl * 4), tpb(N * T * gw * 4),
                         al((size_t)(4 * k.layers + 1) * N * 4), al((size_t)(4 * k.layers + 2) * 4), al((size_t)N * 8),
                         al(16), al((size_t)N * 8), al(T * 8), al(T * 4)};
    for (size_t b : sz) bytes += b;
    cudaError_t e = cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&s->arena, bytes);
    if (e != cudaSuccess) {
        free_session(s);
        return cuda_fail(c, e, "session memory");
    }
    uint8_t *p = (uint8_t *)s->arena;
    int i = 0;
    auto take = [&]() { uint8_t *r = p; p += sz[i++]; return r; };
    s->x = (float *)take();
    s->h = (float *)take();
    s->qkv = (float *)take();
    s->qh = (float *)take();
    s->att = (float *)take();
    s->gu = (float *)take();
    s->a = (float *)take();
    s->logits = (float *)take();
    s->actE = act_q8_carve(take(), (int)T, E);
    s->actF = act_q8_carve(take(), (int)T, F);
    s->tok = (int32_t *)take();
    s->pos = (int64_t *)take();
    s->ids = (int32_t *)take();
    uint8_t *misc = take();
    s->step = (int *)(misc + 16);
    s->attl = (float *)take();
    s->al = (float *)take();
    s->xl = (float *)take();
    s->logl = (float *)take();
    s->gbuf = (float *)take();
    uint8_t *p2p0 = p;
    s->flags = (unsigned *)take();
    s->counters = (unsigned *)take();
    s->keys = (unsigned long long *)take();
    s->epoch = (unsigned *)take();
    s->peer_base = (uint64_t *)take();
    e = cudaMemset(p2p0, 0, (size_t)(p - p2p0));  // flags, counters, epoch start at zero
    s->amax = (unsigned long long *)take();
    s->slot = (int32_t *)take();
    s->slots = slots;
    s->cache_bytes = (size_t)slots * (k.kv_heads / N) * k.context * D * (k.cache_f16 ? 2 : 4);  // this rank's kv heads
    s->kc.resize(k.layers, nullptr);
    s->vc.resize(k.layers, nullptr);
    for (int l = 0; l < k.layers && e == cudaSuccess; l++) {
        e = cudaMalloc(&s->kc[l], s->cache_bytes);
        if (e == cudaSuccess) e = cudaMalloc(&s->vc[l], s->cache_bytes);
    }
    // prompt passes of kAttnPrefillMinRows tokens or more: the many-row attention's score scratch
    const size_t sb = k.max_tokens >= kAttnPrefillMinRows && k.cache_f16 && D == 128
                          ? attn_prefill_scores_bytes((int)k.max_tokens, (int)H, k.kv_heads, k.context)
                          : 0;
    if (e == cudaSuccess && sb) e = cudaMalloc(&s->scores, sb);
    // runs of 16-32 rows (batched steps, short prompts): the records of the
    // tensor-core GEMMs that split K because their matrices have few row
    // tiles (this rank's rows of q|k|v, o, gate|up, down and the head)
    if (e == cudaSuccess && T >= kTcMinRows && k.a8) {
        const int rows = (int)std::min<long long>(T, 32);
        const long long KVl = KV / N;
        auto seg = [](int n) { GemvSeg g{}; g.n = n; return g; };
        const GemvSeg qkv[3] = {seg((int)El), seg((int)KVl), seg((int)KVl)}, o[1] = {seg((int)El)},
                      gu[2] = {seg((int)Fl), seg((int)Fl)}, hd[1] = {seg((int)Vl)};
        size_t need = std::max({gemm_a8_split_bytes(qkv, 3, rows, E), gemm_a8_split_bytes(o, 1, rows, E),
                                gemm_a8_split_bytes(gu, 2, rows, E), gemm_a8_split_bytes(o, 1, rows, F),
                                gemm_a8_split_bytes(hd, 1, rows, E)});
        if (need) {
            e = cudaMalloc(&s->split.rec, need);
            s->split.bytes = need;
        }
    }
    // f32 cos/sin of every position's RoPE angles (float64), for the decode
    // attention's fused RoPE and the step kernel
    const int half = k.rope_dims / 2;
    if (e == cudaSuccess && half > 0) e = cudaMalloc(&s->rope_cs, (size_t)k.context * half * sizeof(float2));
    if (e == cudaSuccess && half > 0) e = launch_rope_table(m->inv_freq, k.context, half, s->rope_cs, s->st);
    if (e == cudaSuccess && k.cache_f16 && D == 128) {
        s->kmap.resize(2 * (size_t)k.layers);  // two per layer: 256- and 128-key boxes
        s->kmap_ok = true;
        for (int l = 0; l < k.layers; l++)
            s->kmap_ok = s->kmap_ok && attn_decode_kmap(s->kc[l], slots, k.kv_heads / N, k.context, &s->kmap[2 * l]);
    }
    if (e != cudaSuccess) {
        free_session(s);
        return cuda_fail(c, e, "key-value cache");
    }
    if ((rc = mimgpu_session_reset(s))) {
        free_session(s);
        return rc;
    }
    if ((rc = setup_step(s))) {
        free_session(s);
        return rc;
    }
    *out = s;
    return MIMGPU_OK;
}

void mimgpu_session_free(mimgpu_session *s) { free_session(s); }

int mimgpu_session_reset(mimgpu_session *s) {
    if (!s) return MIMGPU_EINVAL;
    mimgpu_ctx *c = s->m->ctx;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    int rc = use_device(c);
    if (rc) return rc;
    cudaError_t e = cudaSuccess;
    for (size_t l = 0; l < s->kc.size() && e == cudaSuccess; l++) {
        e = cudaMemsetAsync(s->kc[l], 0, s->cache_bytes, s->st);
        if (e == cudaSuccess) e = cudaMemsetAsync(s->vc[l], 0, s->cache_bytes, s->st);
    }
    if (e == cudaSuccess) e = cudaMemsetAsync(s->amax, 0, sizeof(unsigned long long) * s->m->c.max_tokens, s->st);
    if (e != cudaSuccess) return cuda_fail(c, e, "reset");
    return sync_bounded(c, s->st);
}

int mimgpu_session_run(mimgpu_session *s, const int32_t *tokens, const int64_t *positions, int T, float *logits,
                       int all_rows) {
    if (!s || !tokens || !positions || !logits) return MIMGPU_EINVAL;
    mimgpu_model *m = s->m;
    mimgpu_ctx *c = m->ctx;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    if (T <= 0 || T > m->c.max_tokens) return fail(c, MIMGPU_EINVAL, "%d tokens; the session takes 1..%d", T, m->c.max_tokens);
    for (int i = 0; i < T; i++)
        if (positions[i] < 0 || positions[i] >= m->c.context)
            return fail(c, MIMGPU_EINVAL, "position %lld outside the cache of %d", (long long)positions[i], m->c.context);
    int rc = use_device(c);
    if (rc) return rc;
    cudaError_t e = cudaMemcpyAsync(s->tok, tokens, T * 4, cudaMemcpyHostToDevice, s->st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(s->pos, positions, T * 8, cudaMemcpyHostToDevice, s->st);
    if (e != cudaSuccess) return cuda_fail(c, e, "copy in");
    s->slot0 = 0;
    s->batched = false;
    if (T == 1) {
        if (!s->g_step && (rc = capture(s, false, &s->g_step))) return rc;
        e = cudaGraphLaunch(s->g_step, s->st);
    } else {
        e = enqueue_forward(s, T, all_rows != 0, false, c->status);
    }
    if (e != cudaSuccess) return cuda_fail(c, e, "forward");
    const long long rows = all_rows ? T : 1;
    e = cudaMemcpyAsync(logits, s->logits, rows * m->c.vocab * 4, cudaMemcpyDeviceToHost, s->st);
    if (e != cudaSuccess) return cuda_fail(c, e, "copy out");
    return sync_bounded(c, s->st);
}

int mimgpu_session_generate(mimgpu_session *s, int32_t token, int64_t pos, int steps, int32_t *ids_out) {
    if (!s || !ids_out || steps < 0) return MIMGPU_EINVAL;
    mimgpu_model *m = s->m;
    mimgpu_ctx *c = m->ctx;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    if (steps > 65536 || pos < 0 || pos + steps > m->c.context)
        return fail(c, MIMGPU_EINVAL, "%d steps from position %lld exceed the cache of %d", steps, (long long)pos,
                    m->c.context);
    if (steps == 0) return MIMGPU_OK;
    int rc = use_device(c);
    if (rc) return rc;
    const int zero = 0;
    cudaError_t e = cudaMemcpyAsync(s->tok, &token, 4, cudaMemcpyHostToDevice, s->st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(s->pos, &pos, 8, cudaMemcpyHostToDevice, s->st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(s->step, &zero, 4, cudaMemcpyHostToDevice, s->st);
    if (e != cudaSuccess) return cuda_fail(c, e, "copy in");
    if (!s->g_greedy && (rc = capture(s, true, &s->g_greedy))) return rc;
    for (int i = 0; i < steps && e == cudaSuccess; i++) e = cudaGraphLaunch(s->g_greedy, s->st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(ids_out, s->ids, steps * 4, cudaMemcpyDeviceToHost, s->st);
    if (e != cudaSuccess) return cuda_fail(c, e, "generate");
    return sync_bounded(c, s->st);
}

int mimgpu_session_run_slots(mimgpu_session *s, const int32_t *tokens, const int32_t *slot_ids,
                             const int64_t *positions, int T, float *logits) {
    if (!s || !tokens || !slot_ids || !positions || !logits) return MIMGPU_EINVAL;
    mimgpu_model *m = s->m;
    mimgpu_ctx *c = m->ctx;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    if (T <= 0 || T > m->c.max_tokens) return fail(c, MIMGPU_EINVAL, "%d rows; the session takes 1..%d", T, m->c.max_tokens);
    bool uniform = true;
    for (int i = 0; i < T; i++) {
        if (slot_ids[i] < 0 || slot_ids[i] >= s->slots)
            return fail(c, MIMGPU_EINVAL, "sequence %d of row %d; the session holds %d", slot_ids[i], i, s->slots);
        if (positions[i] < 0 || positions[i] >= m->c.context)
            return fail(c, MIMGPU_EINVAL, "position %lld outside the cache of %d", (long long)positions[i], m->c.context);
        uniform &= slot_ids[i] == slot_ids[0];
    }
    int rc = use_device(c);
    if (rc) return rc;
    cudaError_t e = cudaMemcpyAsync(s->tok, tokens, T * 4, cudaMemcpyHostToDevice, s->st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(s->pos, positions, T * 8, cudaMemcpyHostToDevice, s->st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(s->slot, slot_ids, T * 4, cudaMemcpyHostToDevice, s->st);
    if (e != cudaSuccess) return cuda_fail(c, e, "copy in");
    // rows of one sequence: a prompt pass of that sequence; otherwise one row
    // per sequence, each against its own cache
    s->slot0 = uniform ? slot_ids[0] : 0;
    s->batched = !uniform;
    e = enqueue_forward(s, T, true, false, c->status);
    s->slot0 = 0;
    s->batched = false;
    if (e != cudaSuccess) return cuda_fail(c, e, "forward");
    e = cudaMemcpyAsync(logits, s->logits, (size_t)T * m->c.vocab * 4, cudaMemcpyDeviceToHost, s->st);
    if (e != cudaSuccess) return cuda_fail(c, e, "copy out");
    return sync_bounded(c, s->st);
}

int mimgpu_session_generate_slots(mimgpu_session *s, const int32_t *tokens, const int64_t *positions, int B,
                                  int steps, int32_t *ids_out) {
    if (!s || !tokens || !positions || !ids_out || steps < 0) return MIMGPU_EINVAL;
    mimgpu_model *m = s->m;
    mimgpu_ctx *c = m->ctx;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    if (B < 1 || B > s->slots) return fail(c, MIMGPU_EINVAL, "%d sequences; the session holds %d", B, s->slots);
    if (steps > 65536 || (long long)steps * B > 65536)
        return fail(c, MIMGPU_EINVAL, "%d steps of %d sequences exceed the id buffer", steps, B);
    for (int i = 0; i < B; i++)
        if (positions[i] < 0 || positions[i] + steps > m->c.context)
            return fail(c, MIMGPU_EINVAL, "%d steps from position %lld exceed the cache of %d", steps,
                        (long long)positions[i], m->c.context);
    if (steps == 0) return MIMGPU_OK;
    int rc = use_device(c);
    if (rc) return rc;
    std::vector<int32_t> iota(B);
    for (int i = 0; i < B; i++) iota[i] = i;
    const int zero = 0;
    cudaError_t e = cudaMemcpyAsync(s->tok, tokens, B * 4, cudaMemcpyHostToDevice, s->st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(s->pos, positions, B * 8, cudaMemcpyHostToDevice, s->st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(s->slot, iota.data(), B * 4, cudaMemcpyHostToDevice, s->st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(s->step, &zero, 4, cudaMemcpyHostToDevice, s->st);
    if (e != cudaSuccess) return cuda_fail(c, e, "copy in");
    s->slot0 = 0;
    if (B == 1) {
        if (!s->g_greedy && (rc = capture(s, true, &s->g_greedy))) return rc;
    } else if (s->g_batch_rows != B) {
        if (s->g_batch) cudaGraphExecDestroy(s->g_batch);
        s->g_batch = nullptr;
        s->g_batch_rows = 0;
        if ((rc = capture(s, true, &s->g_batch, B))) return rc;
        s->g_batch_rows = B;
    }
    cudaGraphExec_t g = B == 1 ? s->g_greedy : s->g_batch;
    for (int i = 0; i < steps && e == cudaSuccess; i++) e = cudaGraphLaunch(g, s->st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(ids_out, s->ids, (size_t)steps * B * 4, cudaMemcpyDeviceToHost, s->st);
    if (e != cudaSuccess) return cuda_fail(c, e, "generate");
    return sync_bounded(c, s->st);
}

void *mimgpu_session_stream(mimgpu_session *s) { return s ? (void *)s->st : nullptr; }

int mimgpu_session_set_step_kernel(mimgpu_session *s, int on) {
    if (!s) return MIMGPU_EINVAL;
    mimgpu_ctx *c = s->m->ctx;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    if (on && !s->step_ok) return fail(c, MIMGPU_ENOTHANDLED, "the model does not run through the step kernel");
    if ((on != 0) == s->use_step) return MIMGPU_OK;
    int rc = use_device(c);
    if (rc) return rc;
    cudaStreamSynchronize(s->st);
    if (s->g_step) cudaGraphExecDestroy(s->g_step);
    if (s->g_greedy) cudaGraphExecDestroy(s->g_greedy);
    s->g_step = s->g_greedy = nullptr;
    s->use_step = on != 0;
    return MIMGPU_OK;
}

int mimgpu_session_uses_step_kernel(mimgpu_session *s) { return s && s->use_step ? 1 : 0; }

int mimgpu_session_step_kernels(mimgpu_session *s) { return s ? s->step_kernels : 0; }

namespace {
// the captured graphs carry the old prefetch setting
int drop_graphs(mimgpu_session *s) {
    int rc = use_device(s->m->ctx);
    if (rc) return rc;
    cudaStreamSynchronize(s->st);
    if (s->g_step) cudaGraphExecDestroy(s->g_step);
    if (s->g_greedy) cudaGraphExecDestroy(s->g_greedy);
    if (s->g_batch) cudaGraphExecDestroy(s->g_batch);
    s->g_step = s->g_greedy = s->g_batch = nullptr;
    return MIMGPU_OK;
}
}  // namespace

int mimgpu_session_set_l2_prefetch(mimgpu_session *s, int64_t bytes_per_sm) {
    if (!s || bytes_per_sm < 0 || bytes_per_sm > (1 << 24) || bytes_per_sm % 16) return MIMGPU_EINVAL;
    mimgpu_ctx *c = s->m->ctx;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    int rc = drop_graphs(s);
    if (rc) return rc;
    for (int i = 0; i < 5; i++) {
        s->prefetch_next[i] = (uint32_t)bytes_per_sm;
        s->prefetch_skip[i] = 0;
    }
    return MIMGPU_OK;
}

int mimgpu_session_set_fusions(mimgpu_session *s, unsigned mask) {
    if (!s || (mask & ~MIMGPU_FUSE_NORM)) return MIMGPU_EINVAL;
    mimgpu_ctx *c = s->m->ctx;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    int rc = drop_graphs(s);
    if (rc) return rc;
    s->fuse_norm = (mask & MIMGPU_FUSE_NORM) != 0;
    return MIMGPU_OK;
}

int mimgpu_session_set_l2_prefetch_for(mimgpu_session *s, int kind, int distance, int64_t bytes_per_sm) {
    if (!s || kind < 0 || kind > 4 || distance < 1 || distance > 2 || bytes_per_sm < 0 ||
        bytes_per_sm > (1 << 24) || bytes_per_sm % 16)
        return MIMGPU_EINVAL;
    mimgpu_ctx *c = s->m->ctx;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    int rc = drop_graphs(s);
    if (rc) return rc;
    (distance == 1 ? s->prefetch_next : s->prefetch_skip)[kind] = (uint32_t)bytes_per_sm;
    return MIMGPU_OK;
}

size_t mimgpu_session_trace_bytes(mimgpu_session *s) {
    if (!s || !s->step_ok) return 0;
    return step_trace_words_total(num_sms(), s->m->c.layers) * sizeof(unsigned long long);
}

int mimgpu_session_set_trace(mimgpu_session *s, void *dev_buf, size_t nbytes) {
    if (!s) return MIMGPU_EINVAL;
    mimgpu_ctx *c = s->m->ctx;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    if (dev_buf && nbytes < mimgpu_session_trace_bytes(s))
        return fail(c, MIMGPU_EINVAL, "trace buffer of %zu bytes; the step kernel needs %zu", nbytes,
                    mimgpu_session_trace_bytes(s));
    int rc = use_device(c);
    if (rc) return rc;
    cudaStreamSynchronize(s->st);
    if (s->g_step) cudaGraphExecDestroy(s->g_step);
    if (s->g_greedy) cudaGraphExecDestroy(s->g_greedy);
    s->g_step = s->g_greedy = nullptr;
    s->trace = (unsigned long long *)dev_buf;
    return MIMGPU_OK;
}

int mimgpu_session_ipc_handle(mimgpu_session *s, void *out, size_t nbytes) {
    if (!s || !out || nbytes < sizeof(cudaIpcMemHandle_t)) return MIMGPU_EINVAL;
    mimgpu_ctx *c = s->m->ctx;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    int rc = use_device(c);
    if (rc) return rc;
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, s->arena);
    if (e != cudaSuccess) return cuda_fail(c, e, "ipc handle");
    std::memcpy(out, &h, sizeof(h));
    return MIMGPU_OK;
}

int mimgpu_session_set_peers(mimgpu_session *s, const void *handles, size_t each, int nranks) {
    if (!s || !handles || each < sizeof(cudaIpcMemHandle_t)) return MIMGPU_EINVAL;
    mimgpu_model *m = s->m;
    mimgpu_ctx *c = m->ctx;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    const int N = tp_size(m->tp), k = tp_rank(m->tp);
    if (N < 2 || nranks != N) return fail(c, MIMGPU_EINVAL, "set_peers: %d handles for a group of %d", nranks, N);
    if (s->p2p) return fail(c, MIMGPU_EINVAL, "set_peers: the peers are already mapped");
    int rc = use_device(c);
    if (rc) return rc;
    std::vector<uint64_t> base(N);
    cudaError_t e = cudaSuccess;
    for (int r = 0; r < N && e == cudaSuccess; r++) {
        if (r == k) {
            base[r] = (uint64_t)(uintptr_t)s->arena;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, (const uint8_t *)handles + (size_t)r * each, sizeof(h));
        void *ptr = nullptr;
        e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (e == cudaSuccess) {
            s->opened.push_back(ptr);
            base[r] = (uint64_t)(uintptr_t)ptr;
        }
    }
    if (e == cudaSuccess) e = cudaMemcpy(s->peer_base, base.data(), N * sizeof(uint64_t), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(c, e, "set_peers");
    // graphs captured before now exchange through NCCL; recapture
    if (s->g_step) cudaGraphExecDestroy(s->g_step);
    if (s->g_greedy) cudaGraphExecDestroy(s->g_greedy);
    s->g_step = s->g_greedy = nullptr;
    s->p2p = true;
    return MIMGPU_OK;
}

}  // extern "C"
