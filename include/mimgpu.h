/*
 * mimgpu.h -- C ABI of the B200 (sm_100a) backend for mimir-model's
 * quantized decode hot path.
 *
 * The Go interpreter of gsoultan/mimir-model runs each `call` op through
 * fastPaths[key](attrs, in, dts, shapes) (interp/fast.go:40-59), and those
 * fast paths send the work to internal/kernels.  This library is what a cgo
 * adapter with that signature calls instead.  The entry points below take
 * plain pointers and sizes only; tensors keep the reference's layouts:
 *
 *   - weights: the byte-exact block layouts of spec/dtypes.md (Q8_0 = 64,
 *     Q4_K = 66, Q6_K = 67; F32 = 1, F16 = 2), rows of K elements along the
 *     last axis, W is [N, K] (spec/stdlib.md:216-228);
 *   - activations: f32, row-major, last axis innermost;
 *   - positions: int64; token ids: int32; masks: one byte per bool.
 *
 * Error convention (interp/fast.go:40, interp/interp.go:429-436): every
 * function returns a status code and never aborts or throws across the ABI.
 * MIMGPU_ENOTHANDLED is the fast path's handled=false (a dtype or shape this
 * backend does not serve; the caller runs the canonical body); every other
 * non-zero code is the fast path's err.  mimgpu_last_error() gives the text.
 *
 * Threading: a context may be used from several threads; calls on one
 * context are serialised on its stream.  Weight handles are read-only and
 * may be shared by sessions.  A session is used by one thread at a time.
 */
#ifndef MIMGPU_H
#define MIMGPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MIMGPU_ABI_VERSION 1

enum {
    MIMGPU_OK = 0,
    MIMGPU_ENOTHANDLED = 1, /* not this backend's case: run the canonical body */
    MIMGPU_EINVAL = 2,      /* malformed call (shapes, dtypes, attributes)   */
    MIMGPU_ENOMEM = 3,      /* device memory exhausted                        */
    MIMGPU_ECUDA = 4,       /* CUDA runtime error                             */
    MIMGPU_ENCCL = 5,       /* NCCL error (tensor-parallel sessions)          */
    MIMGPU_ETIMEOUT = 6     /* a bounded wait on the device expired           */
};

enum { MIMGPU_F32 = 1, MIMGPU_F16 = 2, MIMGPU_Q8_0 = 64, MIMGPU_Q4_K = 66, MIMGPU_Q6_K = 67 };

typedef struct mimgpu_ctx mimgpu_ctx;
typedef struct mimgpu_tensor mimgpu_tensor;
typedef struct mimgpu_model mimgpu_model;
typedef struct mimgpu_session mimgpu_session;
typedef struct mimgpu_tp mimgpu_tp;

/* ------------------------------------------------------------ context */

/* ABI version of the loaded library (MIMGPU_ABI_VERSION). */
int mimgpu_abi_version(void);

/* Opens a context on CUDA device `device` with its own stream.  Replaces
 * nothing in the reference (which has no device); the Go side opens one per
 * Program (interp/interp.go:52-67). */
int mimgpu_open(int device, mimgpu_ctx **out);
void mimgpu_close(mimgpu_ctx *ctx);
/* Text of the last error on this context ("" if none).  Valid until the
 * next call on the context. */
const char *mimgpu_last_error(mimgpu_ctx *ctx);
/* Upper bound, in milliseconds, of the waits of this context: a host call
 * waiting for device work (default 60000) and each bounded wait inside a
 * kernel -- on a barrier, a grid counter or a peer's flag -- (default 2000
 * until this is called).  A device wait that runs out ends its kernel early
 * and the call that waits for it returns MIMGPU_ETIMEOUT; the context stays
 * usable. */
int mimgpu_set_timeout_ms(mimgpu_ctx *ctx, int64_t ms);
/* Queues, on `stream` (NULL = the context's stream), a wait until the 32-bit
 * word at `addr` (device or mapped host memory, 4-byte aligned) equals
 * `value`: the device-side doorbell a caller uses to hold this context's work
 * until another process, GPU or the host writes a flag.  No counterpart in
 * the reference.  The wait is bounded by the context's limit
 * (mimgpu_set_timeout_ms); when it runs out, the next call that waits for the
 * device returns MIMGPU_ETIMEOUT. */
int mimgpu_stream_wait_value(mimgpu_ctx *ctx, void *stream, const uint32_t *addr, uint32_t value);

/* ------------------------------------------------------------ weights */

/* Uploads one weight tensor, byte for byte, into device memory.  Called at
 * Open for each weight whose ref.Tensor.Data is a slice of the read-only
 * mapping (interp/interp.go:101-121, file.go:394-399); `bytes` must be
 * exactly the size shape x dtype implies (ref/tensor.go:51-70).  The caller
 * keeps its mapping; the handle owns the device copy. */
int mimgpu_upload(mimgpu_ctx *ctx, int dtype, int ndim, const int64_t *shape, const void *bytes, size_t nbytes,
                  mimgpu_tensor **out);
void mimgpu_tensor_free(mimgpu_tensor *t);
/* Device address of the uploaded bytes (for callers that keep activations
 * on the device). */
const void *mimgpu_tensor_device_ptr(const mimgpu_tensor *t);

/* ------------------------------------------- per-op fast paths (host I/O)
 * Each mirrors one fastPaths entry of interp/fast.go:42-59: inputs and
 * outputs are host buffers; outputs are written by the call. */

/* Dequantize (quant.go:37-69): n elements of dtype from `src` (exactly the
 * bytes they occupy) to f32, bit-exact. */
int mimgpu_dequantize(mimgpu_ctx *ctx, int dtype, const void *src, size_t nbytes, float *dst, int64_t n);

/* dequant_matmul.v1 (fastDequantMatmul, interp/fast.go:222-230):
 * y[rows, N] = x[rows, K] W^T + bias, W decoded exactly; tolerance of
 * spec/stdlib.md section 3.3.  bias may be NULL. */
int mimgpu_dequant_matmul(mimgpu_ctx *ctx, const float *x, int64_t rows, int64_t k, const mimgpu_tensor *w,
                          const float *bias, float *y);

/* dequant_matmul_a8.v2 (fastDequantMatmulA8V2, interp/fast.go:232-244) with
 * its `block` attribute (32 or 256; anything else is EINVAL as in
 * a8Block, interp/transformer.go:201-214), and dequant_matmul_a8.v1
 * (fastDequantMatmulA8, interp/fast.go:225-230) as block 32.  With block 256
 * and Q4_K/Q6_K weights the result is bit-identical to the reference's 8-bit
 * kernels (dotQ8KRef, internal/kernels/q8k_test.go:35-117); with block 32
 * and Q4_K/Q6_K/Q8_0 weights to its AVX2 block-32 kernels (dotQ4KQ8AVX2,
 * dotQ6KQ8AVX2, dotQ8_0Q8AVX2, internal/kernels/kernels_amd64.s:441, 763,
 * 1007; the only block-32 implementation it has).  Rows either refuses take
 * the f32 product (interp/fast.go:282-379); other dtypes take the exact v1
 * product, as the reference does without a kernel (fast.go:254-258). */
int mimgpu_dequant_matmul_a8(mimgpu_ctx *ctx, int block, const float *x, int64_t rows, int64_t k,
                             const mimgpu_tensor *w, const float *bias, float *y);

/* rms_norm.v1 over the last axis (fastRMSNorm, interp/fast.go:434-485). */
int mimgpu_rms_norm(mimgpu_ctx *ctx, const float *x, int64_t rows, int64_t n, const float *scale, double eps,
                    float *y);

/* rope.v1 (fastRope, interp/fast.go:507-557) on x [B,H,T,D] with positions
 * [pos_rows, T] (pos_rows 1 or B); YaRN attributes are not served
 * (ENOTHANDLED). */
int mimgpu_rope(mimgpu_ctx *ctx, const float *x, int b, int h, int t, int d, const int64_t *pos, int pos_rows,
                double theta, int rotary_dims, int interleaved, float *y);

/* attention.v1 / v2 (attentionFast, interp/fast.go:569-751): q f32
 * [B,Hq,Tq,D]; k, v [B,Hkv,Tk,D] of kv_dtype F32 or F16; optional boolean
 * mask (one byte per element) of shape mask_shape[4], each axis 1 or full.
 * scale <= 0 means 1/sqrt(D).  Float masks and softcap are ENOTHANDLED. */
int mimgpu_attention(mimgpu_ctx *ctx, const float *q, int b, int hq, int tq, int d, const void *k, const void *v,
                     int kv_dtype, int hkv, int tk, const uint8_t *mask, const int *mask_shape, double scale,
                     int causal, float *out);

/* swiglu.v1 (fastSwiglu, interp/fast.go:487-498): y = silu(a) * b. */
int mimgpu_swiglu(mimgpu_ctx *ctx, const float *a, const float *b, int64_t n, float *y);

/* embedding.v1 (fastEmbedding, interp/fast.go:818-842): decoded rows of
 * `table` for n int32 ids; out-of-range ids give zero rows. */
int mimgpu_embedding(mimgpu_ctx *ctx, const mimgpu_tensor *table, const int32_t *ids, int64_t n, float *y);

/* ------------------------------- device-resident products (no host copies)
 * Same arithmetic as the host-buffer calls; all pointers are device memory
 * and the work is queued on `stream` (a cudaStream_t, NULL = the context's
 * stream) without waiting.  Used by callers that keep activations in HBM.
 * These calls return before the work runs, so a bounded device wait of
 * theirs that runs out is reported (MIMGPU_ETIMEOUT) by the next call on the
 * same context that waits for the device: any host-buffer call or session
 * run. */
int mimgpu_dequant_matmul_a8_dev(mimgpu_ctx *ctx, void *stream, const float *x_dev, int64_t rows, int64_t k,
                                 const mimgpu_tensor *w, const float *bias_dev, float *y_dev);
int mimgpu_dequant_matmul_dev(mimgpu_ctx *ctx, void *stream, const float *x_dev, int64_t rows, int64_t k,
                              const mimgpu_tensor *w, const float *bias_dev, float *y_dev);
/* mimgpu_dequant_matmul_a8_dev with the block attribute of
 * mimgpu_dequant_matmul_a8 (32 or 256; mimgpu_dequant_matmul_a8_dev is
 * block 256). */
int mimgpu_dequant_matmul_a8_block_dev(mimgpu_ctx *ctx, void *stream, int block, const float *x_dev, int64_t rows,
                                       int64_t k, const mimgpu_tensor *w, const float *bias_dev, float *y_dev);

/* Same as mimgpu_dequant_matmul_a8_dev for Q4_K / Q6_K weights with K a
 * multiple of 256, but the 8-bit activation scratch lives in a fixed 1 MiB
 * static device array instead of the context's workspace, so the call
 * allocates no device memory.  No counterpart in the reference: it serves
 * callers that cannot allocate while they run (a server whose HBM is all
 * handed to its own pool, a decode loop that cannot afford the device-wide
 * synchronization of cudaMalloc / cudaFree).
 * Limit: rows x K must fit the buffer (act bytes <= 1 MiB, e.g. 16 rows of
 * 14336); larger calls return MIMGPU_EINVAL with the sizes in the message.
 * Other dtypes return MIMGPU_ENOTHANDLED.  The first call on a device looks
 * the buffer's address up (cudaGetSymbolAddress), so make it outside stream
 * capture.  The buffer is shared by every call on a device: two calls whose
 * work overlaps in time on that device (different streams, or different
 * contexts, without ordering between them) race on it; order them. */
int mimgpu_dequant_matmul_a8_static(mimgpu_ctx *ctx, void *stream, const float *x_dev, int64_t rows, int64_t k,
                                    const mimgpu_tensor *w, const float *bias_dev, float *y_dev);

/* ------------------------------------------ 8-bit activations on the device
 * Rows of activations quantized once and multiplied by several weights, as
 * linearA8 does with a Q8Batch (interp/fast.go:282-379, internal/kernels/
 * q8.go:154-201).  Blocks of 256 (dequant_matmul_a8.v2, block = 256). */
typedef struct mimgpu_q8 mimgpu_q8;
int mimgpu_q8_new(mimgpu_ctx *ctx, int64_t rows, int64_t k, mimgpu_q8 **out);
void mimgpu_q8_free(mimgpu_q8 *q);
/* QuantizeBlocks (q8.go:50-97) of rows x k f32 device values; rows the
 * reference refuses are flagged and later take the f32 product. */
int mimgpu_q8_quantize_dev(mimgpu_ctx *ctx, void *stream, const float *x_dev, mimgpu_q8 *q);
/* y = x W^T (+ bias) from activations quantized by mimgpu_q8_quantize_dev
 * (DotQ8 / DotQ8x4, q8.go:119-235); x_dev is the same f32 input, read only
 * for refused rows.  W must be Q4_K or Q6_K. */
int mimgpu_gemv_q8_dev(mimgpu_ctx *ctx, void *stream, const mimgpu_q8 *q, const float *x_dev,
                       const mimgpu_tensor *w, const float *bias_dev, float *y_dev);

/* The same product for n (1..4) matrices sharing the activations, in one
 * launch: ys[i] = x ws[i]^T, as the decode step runs q|k|v and gate|up (the
 * reference runs them as separate calls of linearA8, interp/fast.go:282-379,
 * with the same per-matrix bits). */
int mimgpu_gemv_q8_fused_dev(mimgpu_ctx *ctx, void *stream, const mimgpu_q8 *q, const float *x_dev, int n,
                             const mimgpu_tensor *const *ws, float *const *ys);

/* ------------------------------------------------ synthetic weights, bytes
 * Not part of the reference interface: seeded random-init weights for the
 * benchmark configurations, made on the device (values from N(mean, sigma)
 * by a counter-based generator, encoded as dtype), and a copy of a tensor's
 * bytes back to the host. */
int mimgpu_synth_tensor(mimgpu_ctx *ctx, int dtype, uint64_t seed, int ndim, const int64_t *shape, float mean,
                        float sigma, mimgpu_tensor **out);
/* Rows [row0, row0 + shape[0]) of the tensor mimgpu_synth_tensor makes with the
 * same seed (a tensor-parallel rank's shard, byte for byte). */
int mimgpu_synth_rows(mimgpu_ctx *ctx, int dtype, uint64_t seed, int ndim, const int64_t *shape, int64_t row0,
                      float mean, float sigma, mimgpu_tensor **out);
int mimgpu_tensor_download(const mimgpu_tensor *t, void *bytes, size_t nbytes);
size_t mimgpu_tensor_nbytes(const mimgpu_tensor *t);

/* ----------------------------------------- whole-step decoder (sessions)
 * The llama graph of importer/llama.go:317-547 run as one device-resident
 * step per Session.Run (interp/interp.go:409-526): activations and the
 * key-value cache stay in HBM; only token ids, positions and the logits (or
 * the greedy id) cross the bus. */
typedef struct {
    int layers, embed, ffn, heads, kv_heads, head_dim, rope_dims, vocab;
    int context;      /* key-value cache length C per sequence */
    double rope_theta, norm_eps;
    int a8;           /* 1: dequant_matmul_a8.v2 block 256 for Q4_K/Q6_K weights */
    int cache_f16;    /* 1: f16 cache (attention.v2); 0: f32 cache (attention.v1) */
    int interleaved;  /* rope pairs: 1 adjacent (llama), 0 halves (qwen2) */
    int max_tokens;   /* largest T of one run (prompt length) */
} mimgpu_llama_config;

int mimgpu_model_new(mimgpu_ctx *ctx, const mimgpu_llama_config *cfg, mimgpu_model **out);
/* Binds an uploaded weight by its GGUF name (token_embd.weight,
 * blk.N.attn_q.weight, ..., output_norm.weight, output.weight, and for a
 * Qwen 2 graph the f32 biases blk.N.attn_q.bias / attn_k.bias / attn_v.bias,
 * all three or none: the optional third input of the q, k, v products,
 * importer/llama.go:470-478).  The model keeps the handle; it must outlive
 * the model. */
int mimgpu_model_set_weight(mimgpu_model *m, const char *name, const mimgpu_tensor *w);
void mimgpu_model_free(mimgpu_model *m);

int mimgpu_session_new(mimgpu_model *m, mimgpu_session **out);
void mimgpu_session_free(mimgpu_session *s);
/* Zeroes the key-value cache (a fresh Session). */
int mimgpu_session_reset(mimgpu_session *s);
/* One run of the graph: T tokens at the given positions, logits [T, vocab]
 * (all_rows) or the last row's [vocab] into host memory, as
 * cmd/mim-run/main.go:133-174 reads them. */
int mimgpu_session_run(mimgpu_session *s, const int32_t *tokens, const int64_t *positions, int t, float *logits,
                       int all_rows);
/* Greedy decode (cmd/mim-run/main.go:219-257): feeds `token` at `pos`, picks
 * the first maximum of the logits, feeds it back, `steps` times; writes the
 * picked ids.  One step is one device-resident graph launch. */
int mimgpu_session_generate(mimgpu_session *s, int32_t token, int64_t pos, int steps, int32_t *ids_out);
/* Batched decoding (no counterpart in the reference, whose sessions hold one
 * sequence): a session of `slots` independent sequences, each with its own
 * key-value cache (1 <= slots <= max_tokens).  mimgpu_session_new is
 * mimgpu_session_new_slots(m, 1, out). */
int mimgpu_session_new_slots(mimgpu_model *m, int slots, mimgpu_session **out);
/* One run of t rows, row i token tokens[i] of sequence slot_ids[i] at
 * positions[i]; logits [t, vocab].  Rows all of one sequence are a prompt
 * pass of that sequence; otherwise each row attends to its own sequence's
 * cache.  Every row's logits are the bits a single-sequence session gives. */
int mimgpu_session_run_slots(mimgpu_session *s, const int32_t *tokens, const int32_t *slot_ids,
                             const int64_t *positions, int t, float *logits);
/* Greedy decode of sequences 0..b-1 together: sequence i is fed tokens[i] at
 * positions[i], then its own picks, `steps` times; ids_out [steps][b].  One
 * step of all b sequences is one device-resident graph launch. */
int mimgpu_session_generate_slots(mimgpu_session *s, const int32_t *tokens, const int64_t *positions, int b,
                                  int steps, int32_t *ids_out);
/* The session's CUDA stream (a cudaStream_t), for callers that time or
 * order their own device work against the session's. */
void *mimgpu_session_stream(mimgpu_session *s);
/* How one-token steps of sequence 0 run (mimgpu_session_run with t = 1,
 * mimgpu_session_generate; no counterpart in the reference, whose Session.Run
 * interprets the graph op by op, interp/interp.go:409-526): on = 1 runs the
 * whole step as one persistent kernel that streams every layer's weights
 * through one pipeline; on = 0 (the default) launches one kernel per op, which
 * measured faster on B200 (8B shape 2.08 vs 2.45 ms per token).  Both give the
 * same bits.  The persistent kernel serves single-GPU sessions of
 * 8-bit-activation models with Q4_K / Q6_K matrices, E and F multiples of 256
 * (E 2048..8192, F 2048..32768), head size 128, an f16 cache and interleaved
 * RoPE; for other
 * models on = 1 returns MIMGPU_ENOTHANDLED. */
int mimgpu_session_set_step_kernel(mimgpu_session *s, int on);
/* 1 when one-token steps run as one persistent kernel, else 0. */
int mimgpu_session_uses_step_kernel(mimgpu_session *s);

/* L2 prefetch between the one-token GEMVs of a decode step: once a GEMV has
 * issued its own weight copies, each SM prefetches into L2 the first
 * `bytes_per_sm` of its slab of the next GEMV's matrices (a multiple of 16,
 * at most 16 MiB; 0 turns it off; default 160 KiB), so that the next GEMV
 * starts from L2 while HBM would otherwise idle through the launch boundary
 * and the small kernels between.  Results are unchanged. */
int mimgpu_session_set_l2_prefetch(mimgpu_session *s, int64_t bytes_per_sm);
/* The same per GEMV kind and distance: `kind` is the GEMV prefetched (0 the
 * q|k|v GEMV, 1 o, 2 gate|up, 3 down, 4 the head), `distance` 1 when the
 * GEMV just before it issues the prefetch, 2 when the one before that does
 * (for instance the q|k|v GEMV prefetching gate|up bytes that stream while
 * the attention runs).  mimgpu_session_set_l2_prefetch sets every kind at
 * distance 1 and clears distance 2.  Results are unchanged. */
int mimgpu_session_set_l2_prefetch_for(mimgpu_session *s, int kind, int distance, int64_t bytes_per_sm);

/* Which small ops a one-token step on one GPU runs inside a GEMV instead of
 * as kernels of their own (default: all): MIMGPU_FUSE_NORM, each rms_norm in
 * the prologue of the GEMV that reads it.  Results are unchanged, bit for
 * bit; the flag exists to compare the forms. */
#define MIMGPU_FUSE_NORM 1u
int mimgpu_session_set_fusions(mimgpu_session *s, unsigned mask);

/* Kernel launches in one replay of the session's captured one-token greedy
 * step (mimgpu_session_generate), counted from the CUDA graph; 0 before the
 * first capture. */
int mimgpu_session_step_kernels(mimgpu_session *s);
/* Profiling: with a device buffer of mimgpu_session_trace_bytes(s) bytes
 * bound, every persistent-kernel step writes its phase timeline there (per
 * CTA, %globaltimer nanoseconds: start, end, and per op the moments its
 * activation was ready and staged, its stages consumed and chained, and its
 * first and last weight stage issued; the slot layout is documented in the
 * repository's step.h).  NULL unbinds.  The size is 0 when the session does
 * not use the persistent kernel. */
size_t mimgpu_session_trace_bytes(mimgpu_session *s);
int mimgpu_session_set_trace(mimgpu_session *s, void *dev_buf, size_t nbytes);

/* ------------------------------------------------- tensor parallelism
 * No counterpart in the reference (one process on CPU).  Ranks of one node,
 * one process and context per GPU, share an NCCL communicator (NCCL is
 * loaded at run time).  With a group of N bound, rank k computes, as complete
 * block-ordered dot products, the q|k|v rows of its query heads
 * [kH/N, (k+1)H/N) and kv heads [kHkv/N, (k+1)Hkv/N) (RoPE, its key-value
 * cache and attention on those heads only), o rows [kE/N, (k+1)E/N) after an
 * exchange of the attention output, gate/up rows [kF/N, (k+1)F/N), down rows
 * [kE/N, (k+1)E/N) after an exchange of the SwiGLU output, and its vocabulary
 * rows; the residual is exchanged after o and after down.  Every rank
 * produces the single-GPU logits and greedy ids bit for bit.  A weight bound
 * with mimgpu_model_set_weight is either the full tensor (the rank reads its
 * rows) or exactly this rank's rows (its shard: no rank then holds another's
 * bytes).  Needs heads, kv heads and ffn divisible by N. */
/* Rank 0 makes the group id (NCCL_UNIQUE_ID_BYTES = 128 bytes) and hands it
 * to the others. */
int mimgpu_tp_unique_id(void *id, size_t nbytes);
int mimgpu_tp_new(mimgpu_ctx *ctx, const void *id, size_t nbytes, int nranks, int rank, mimgpu_tp **out);
void mimgpu_tp_free(mimgpu_tp *tp);
/* Binds the group before the model's first session; the group must outlive
 * the model's sessions. */
int mimgpu_model_set_tp(mimgpu_model *m, mimgpu_tp *tp);
/* Peer-memory exchanges for the one-token step: every rank exports its
 * session's device arena (a cudaIpcMemHandle_t, 64 bytes), the handles are
 * all-gathered by the caller (rank order) and handed to every rank's
 * session.  From then on the SwiGLU output, the residual columns and the
 * argmax keys of a decode step travel over NVLink inside the kernels that
 * produce them (stores into every rank's copy, an epoch flag per exchange,
 * bounded waits), with no collective launches; multi-token runs keep the
 * NCCL all-gathers. */
int mimgpu_session_ipc_handle(mimgpu_session *s, void *out, size_t nbytes);
int mimgpu_session_set_peers(mimgpu_session *s, const void *handles, size_t each, int nranks);

#ifdef __cplusplus
}
#endif
#endif /* MIMGPU_H */
