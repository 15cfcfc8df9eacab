/*
 * mimoracle.h -- CPU restatement of the mimir-model quantized decode path.
 *
 * TEST INFRASTRUCTURE, NOT PRODUCT.  Only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline / --impl reference legs may load this code,
 * and only as the checker or as the timed CPU baseline.  The GPU library
 * (libmimgpu.so) never links or calls it.
 *
 * Every function restates one piece of the Go reference (gsoultan/mimir-model)
 * and cites the file:line it follows.  Paths are relative to that project.
 *
 * Arithmetic contract: this file is compiled with -ffp-contract=off so that a
 * product followed by a sum is rounded twice, as the Go code computes it on
 * amd64; fused multiply-adds appear only where the reference's kernels use
 * one (fmaf in mo_dot_q8k_ref after internal/kernels/q8k_test.go:35-117, and
 * in the restated amd64 attention and SiLU kernels of attn_amd64.s).
 */
#ifndef MIMORACLE_H
#define MIMORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* dtype ids, spec/dtypes.md:124-135 and dtype.go:25-43 */
enum { MO_F32 = 1, MO_F16 = 2, MO_Q8_0 = 64, MO_Q4_K = 66, MO_Q6_K = 67 };

/* ---- scalar conversions, float.go:24-88 ---- */
float mo_f16_to_f32(uint16_t h);
uint16_t mo_f32_to_f16(float f);

/* Bytes of one row of k elements of dtype dt; 0 when k is not a multiple of
 * the block size or dt is not one of the dtypes above. dtype.go:48-129 */
int64_t mo_row_bytes(int dt, int64_t k);

/* ---- block decode, quant.go:37-69 (Dequantize), 197-344 ----
 * Returns 0, or -1 for an unsupported dtype or a length that is not a
 * multiple of the block size. */
int mo_dequantize(int dt, const uint8_t *src, float *dst, int64_t n);

/* ---- encoders ----
 * Q8_0 follows quant.go:208-228 (ggml's reference quantizer).  The
 * reference has no Q4_K/Q6_K encoder; these two are this project's own,
 * non-normative (spec/dtypes.md says encoders are not part of the format),
 * and produce blocks in the layouts quant.go:274-344 decodes. */
void mo_quantize_q8_0(const float *x, uint8_t *dst, int64_t n);
void mo_quantize_q4_k(const float *x, uint8_t *dst, int64_t n);
void mo_quantize_q6_k(const float *x, uint8_t *dst, int64_t n);
int mo_quantize(int dt, const float *x, uint8_t *dst, int64_t n);

/* Seeded synthetic weights: n*k values from N(0, sigma) (a counter-based
 * generator keyed by seed, so any row range can be produced independently),
 * encoded as dt into dst (n rows of mo_row_bytes(dt,k) bytes). */
int mo_gen_weight(int dt, uint64_t seed, int64_t n, int64_t k, float sigma, uint8_t *dst, int nthreads);
/* Rows [row0, row0 + n) of the tensor mo_gen_weight makes with the same seed. */
int mo_gen_weight_rows(int dt, uint64_t seed, int64_t row0, int64_t n, int64_t k, float sigma, uint8_t *dst,
                       int nthreads);
/* n values from N(mean, sigma) into x (f32), same generator. */
void mo_gen_normal(uint64_t seed, int64_t n, float mean, float sigma, float *x);

/* ---- 8-bit activations, internal/kernels/q8.go:50-97, 237-273 ----
 * Quantizes x[0..k) in blocks of `block` (32 or 256).  q gets k int8, d32
 * k/32 scales (the block's d repeated per run of 32), xs k/32 sums, m32 k/2
 * pair sums.  Returns 1, or 0 when the reference refuses (NaN, |x| > 2^60,
 * bad length or block); the caller then uses the f32 kernels. */
int mo_q8_quantize(const float *x, int64_t k, int block, int8_t *q, float *d32, int16_t *xs, int16_t *m32);

/* dotQ8KRef, internal/kernels/q8k_test.go:35-117: the exact integer block
 * sums of a Q4_K or Q6_K row against 8-bit activations in blocks of 256,
 * then one fused multiply-add per block in block order.  Returns 1 and sets
 * *out, or 0 when a block scale of the row is not finite. */
int mo_dot_q8k_ref(int dt, const uint8_t *row, const int8_t *q, const float *d32, const int16_t *xs, int64_t k, float *out);
/* Its exact integer block sums as the reference computes them on amd64, in
 * AVX2 (default when compiled for AVX2), or by the scalar loops (0): the
 * same bits either way.  mo_simd_active() says which runs. */
void mo_set_simd(int on);
int mo_simd_active(void);

/* RowDot.DotQ8 with blocks of 32 (q8.go:143-151): the AVX2 kernels
 * dotQ4KQ8AVX2, dotQ6KQ8AVX2 and dotQ8_0Q8AVX2 (internal/kernels/
 * kernels_amd64.s:441, 763, 1007) restated lane by lane for a Q4_K, Q6_K or
 * Q8_0 row against activations quantized with block 32.  Returns 1 and sets
 * *out, or 0 when a block scale of the row is not finite. */
int mo_dot_q8_b32(int dt, const uint8_t *row, const int8_t *q, const float *d32, const int16_t *xs, int64_t k,
                  float *out);

/* dotF32Go, internal/kernels/kernels.go:46-62: four strided accumulators. */
float mo_dot_f32(const float *a, const float *b, int64_t n);

/* ---- composites (interp/fast.go) ---- */
/* dequant_matmul.v1, interp/fast.go:160-224: y[rows,n] = x[rows,k] w^T + bias.
 * Rows of w are decoded exactly (Dequantize) and dotted with dotF32Go. */
int mo_dequant_matmul(const float *x, int64_t rows, int64_t k, int dt, const uint8_t *w, int64_t n,
                      const float *bias, float *y, int nthreads);
/* dequant_matmul_a8.v1 (block 32) and .v2 (block 256), interp/fast.go:
 * 238-379 (linearA8): each row of x is quantized once; rows or weight rows
 * the 8-bit kernels refuse go through the f32 path.  Blocks of 256 take
 * Q4_K/Q6_K (dotQ8KRef), blocks of 32 Q4_K/Q6_K/Q8_0 (mo_dot_q8_b32); other
 * dtypes use the f32 path, as the reference does without a kernel. */
int mo_dequant_matmul_a8(const float *x, int64_t rows, int64_t k, int dt, const uint8_t *w, int64_t n,
                         const float *bias, int block, float *y, int nthreads);

/* rms_norm.v1 fast path, interp/fast.go:434-485. */
void mo_rms_norm(const float *x, int64_t rows, int64_t n, const float *scale, double eps, float *y);
/* rope.v1 fast path, interp/fast.go:507-557 (+ readRope, interp/transformer.go:257-326,
 * without YaRN).  pos has pos_rows (1 or B) rows of T positions. */
int mo_rope(const float *x, int B, int H, int T, int D, const int64_t *pos, int pos_rows, double theta,
            int rotary, int interleaved, float *y);
/* attention.v1/v2 fast path, interp/fast.go:569-751 with the amd64 kernels of
 * internal/kernels/attn.go:26-121 / attn_amd64.s (rows with a masked key
 * inside their visible range take the scalar path of fast.go:661-716).  k and v are f32 or f16 (kv_dtype) [B,Hkv,Tk,D]; mask is
 * NULL or bool bytes broadcast over mask_shape[4] (each 1 or full).  Rows
 * whose keys are all masked give NaN. */
int mo_attention(const float *q, int B, int Hq, int Tq, int D, const void *k, const void *v, int kv_dtype,
                 int Hkv, int Tk, const uint8_t *mask, const int *mask_shape, double scale, int causal,
                 float *out);
/* swiglu.v1 fast path, interp/fast.go:487-498 with kernels/attn.go:63-73
 * (siluMulF32AVX2 for the first n&~7 elements, float64 for the rest). */
void mo_swiglu(const float *a, const float *b, int64_t n, float *y);
/* embedding.v1 fast path, interp/fast.go:818-842; out-of-range ids give zeros. */
int mo_embedding(int dt, const uint8_t *table, int64_t V, int64_t E, const int32_t *ids, int64_t n, float *y);
/* greedy pick, cmd/mim-run/main.go:184-193: first index of the maximum. */
int32_t mo_argmax(const float *v, int64_t n);
/* RNE f32 -> f16 of n values (the cast before the cache scatter). */
void mo_cast_f16(const float *x, uint16_t *y, int64_t n);

/* ---- the llama graph, importer/llama.go:317-547, run one op at a time ---- */
typedef struct {
    int layers, embed, ffn, heads, kv_heads, head_dim, rope_dims, vocab, context;
    double rope_theta, norm_eps;
    int a8;       /* 1: dequant_matmul_a8.v2 block 256 for Q4_K/Q6_K (importer/llama.go:264-280) */
    int cache_f16;/* 1: f16 cache + attention.v2; 0: f32 cache + attention.v1 */
    int interleaved; /* 1 for llama (adjacent pairs), 0 for qwen2 */
    int nthreads;
} mo_llama_config;

typedef struct mo_llama mo_llama;
mo_llama *mo_llama_new(const mo_llama_config *c);
void mo_llama_free(mo_llama *m);
/* Registers a weight by its GGUF name (token_embd.weight, blk.N.attn_q.weight,
 * output.weight, ...).  The bytes are not copied and must outlive m. */
int mo_llama_set_weight(mo_llama *m, const char *name, int dt, const void *data);
/* Zeroes the key-value cache. */
void mo_llama_reset(mo_llama *m);
/* Runs T tokens at the given positions (one Session.Run of the graph) and
 * writes logits [T, vocab] (all_rows) or only the last row's [vocab]. */
int mo_llama_forward(mo_llama *m, const int32_t *tokens, const int64_t *positions, int T, float *logits, int all_rows);

#ifdef __cplusplus
}
#endif
#endif
