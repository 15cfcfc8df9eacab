/*
 * capi_driver.c -- the C ABI of include/mimgpu.h driven from plain C, the
 * way a cgo binding in the Go interpreter would call it (no Python, no
 * ctypes), checked against the CPU restatement of the reference (oracle/,
 * test infrastructure linked only here).
 *
 *   1. dequant_matmul_a8.v2 (block 256) of one and of 24 activation rows
 *      through mimgpu_dequant_matmul_a8 with host buffers, bit for bit with
 *      the reference's 8-bit kernels (dotQ8KRef, internal/kernels/
 *      q8k_test.go:35-117 of gsoultan/mimir-model);
 *   2. a malformed call returns MIMGPU_EINVAL with a message, and the
 *      context keeps working (interp/fast.go:40: err, not a crash);
 *   3. a two-layer Llama uploaded tensor by tensor and bound by GGUF name
 *      (what interp.Load does with File.TensorData, interp/interp.go:101-121),
 *      a 12-token prompt through mimgpu_session_run (logits bit-identical to
 *      the oracle's), then 8 greedy tokens through mimgpu_session_generate,
 *      identical to the oracle's greedy loop (cmd/mim-run/main.go:219-257).
 *
 * Exit status 0 and "capi driver ok" on success; tests/test_capi_c.py builds
 * and runs it.
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "mimgpu.h"
#include "mimoracle.h"

#define CHECK(cond, ...)                      \
    do {                                      \
        if (!(cond)) {                        \
            fprintf(stderr, "FAIL: " __VA_ARGS__); \
            fprintf(stderr, "\n");            \
            exit(1);                          \
        }                                     \
    } while (0)

static int same_bits(const float *a, const float *b, size_t n) { return memcmp(a, b, n * sizeof(float)) == 0; }

static void *xmalloc(size_t n) {
    void *p = malloc(n ? n : 1);
    CHECK(p != NULL, "out of host memory");
    return p;
}

/* 1 and 2: the per-op fast path with host buffers */
static void check_matmul(mimgpu_ctx *ctx) {
    const int64_t n = 512, k = 4096;
    const int64_t rb = mo_row_bytes(MIMGPU_Q4_K, k);
    uint8_t *w = xmalloc((size_t)(n * rb));
    CHECK(mo_gen_weight(MIMGPU_Q4_K, 41, n, k, 0.02f, w, 4) == 0, "gen weight");
    mimgpu_tensor *t = NULL;
    const int64_t shape[2] = {n, k};
    CHECK(mimgpu_upload(ctx, MIMGPU_Q4_K, 2, shape, w, (size_t)(n * rb), &t) == MIMGPU_OK, "upload: %s",
          mimgpu_last_error(ctx));
    const int64_t rows_list[2] = {1, 24};
    for (int c = 0; c < 2; c++) {
        const int64_t rows = rows_list[c];
        float *x = xmalloc((size_t)(rows * k) * sizeof(float));
        float *got = xmalloc((size_t)(rows * n) * sizeof(float));
        float *want = xmalloc((size_t)(rows * n) * sizeof(float));
        mo_gen_normal(42 + (uint64_t)c, rows * k, 0.f, 1.f, x);
        CHECK(mimgpu_dequant_matmul_a8(ctx, 256, x, rows, k, t, NULL, got) == MIMGPU_OK, "a8 matmul: %s",
              mimgpu_last_error(ctx));
        CHECK(mo_dequant_matmul_a8(x, rows, k, MIMGPU_Q4_K, w, n, NULL, 256, want, 4) == 0, "oracle matmul");
        CHECK(same_bits(got, want, (size_t)(rows * n)), "a8 matmul of %lld rows differs from dotQ8KRef",
              (long long)rows);
        free(x);
        free(got);
        free(want);
    }
    /* a block attribute the reference refuses (a8Block, interp/transformer.go:201-214) */
    float x1[4096], y1[512];
    memset(x1, 0, sizeof(x1));
    CHECK(mimgpu_dequant_matmul_a8(ctx, 64, x1, 1, k, t, NULL, y1) == MIMGPU_EINVAL, "block 64 accepted");
    CHECK(strlen(mimgpu_last_error(ctx)) > 0, "no error text");
    CHECK(mimgpu_dequant_matmul_a8(ctx, 256, x1, 1, k, t, NULL, y1) == MIMGPU_OK, "context unusable after EINVAL");
    mimgpu_tensor_free(t);
    free(w);
}

/* 3: a whole model through the session calls */
enum { L = 2, E = 512, H = 4, HKV = 2, D = 128, F = 1024, V = 1000, P = 12, STEPS = 8, C = 64 };

typedef struct {
    char name[64];
    int dt;
    int64_t rows, cols; /* cols 0: a vector */
    void *bytes;
    size_t nbytes;
} weight;

static void make_weight(weight *w, const char *name, int dt, int64_t rows, int64_t cols, uint64_t seed) {
    snprintf(w->name, sizeof(w->name), "%s", name);
    w->dt = dt;
    w->rows = rows;
    w->cols = cols;
    if (dt == MIMGPU_F32) {
        w->nbytes = (size_t)rows * sizeof(float);
        w->bytes = xmalloc(w->nbytes);
        mo_gen_normal(seed, rows, 1.f, 0.02f, (float *)w->bytes);
    } else {
        w->nbytes = (size_t)(rows * mo_row_bytes(dt, cols));
        w->bytes = xmalloc(w->nbytes);
        CHECK(mo_gen_weight(dt, seed, rows, cols, 0.02f, (uint8_t *)w->bytes, 4) == 0, "gen %s", name);
    }
}

static void check_model(mimgpu_ctx *ctx) {
    weight ws[3 + 9 * L];
    int nw = 0;
    uint64_t seed = 7000;
    char nm[64];
    make_weight(&ws[nw++], "token_embd.weight", MIMGPU_Q4_K, V, E, seed++);
    for (int l = 0; l < L; l++) {
        snprintf(nm, sizeof(nm), "blk.%d.attn_norm.weight", l);
        make_weight(&ws[nw++], nm, MIMGPU_F32, E, 0, seed++);
        snprintf(nm, sizeof(nm), "blk.%d.attn_q.weight", l);
        make_weight(&ws[nw++], nm, MIMGPU_Q4_K, E, E, seed++);
        snprintf(nm, sizeof(nm), "blk.%d.attn_k.weight", l);
        make_weight(&ws[nw++], nm, MIMGPU_Q4_K, HKV * D, E, seed++);
        snprintf(nm, sizeof(nm), "blk.%d.attn_v.weight", l);
        make_weight(&ws[nw++], nm, MIMGPU_Q6_K, HKV * D, E, seed++);
        snprintf(nm, sizeof(nm), "blk.%d.attn_output.weight", l);
        make_weight(&ws[nw++], nm, MIMGPU_Q4_K, E, E, seed++);
        snprintf(nm, sizeof(nm), "blk.%d.ffn_norm.weight", l);
        make_weight(&ws[nw++], nm, MIMGPU_F32, E, 0, seed++);
        snprintf(nm, sizeof(nm), "blk.%d.ffn_gate.weight", l);
        make_weight(&ws[nw++], nm, MIMGPU_Q4_K, F, E, seed++);
        snprintf(nm, sizeof(nm), "blk.%d.ffn_up.weight", l);
        make_weight(&ws[nw++], nm, MIMGPU_Q4_K, F, E, seed++);
        snprintf(nm, sizeof(nm), "blk.%d.ffn_down.weight", l);
        make_weight(&ws[nw++], nm, MIMGPU_Q6_K, E, F, seed++);
    }
    make_weight(&ws[nw++], "output_norm.weight", MIMGPU_F32, E, 0, seed++);
    make_weight(&ws[nw++], "output.weight", MIMGPU_Q6_K, V, E, seed++);

    /* the GPU side: upload every tensor, bind it by name */
    const mimgpu_llama_config cfg = {L, E, F, H, HKV, D, D, V, C, 500000.0, 1e-5, 1, 1, 1, P};
    mimgpu_model *m = NULL;
    CHECK(mimgpu_model_new(ctx, &cfg, &m) == MIMGPU_OK, "model_new: %s", mimgpu_last_error(ctx));
    mimgpu_tensor *ts[3 + 9 * L];
    for (int i = 0; i < nw; i++) {
        const int64_t shape[2] = {ws[i].rows, ws[i].cols};
        CHECK(mimgpu_upload(ctx, ws[i].dt, ws[i].cols ? 2 : 1, shape, ws[i].bytes, ws[i].nbytes, &ts[i]) ==
                  MIMGPU_OK,
              "upload %s: %s", ws[i].name, mimgpu_last_error(ctx));
        CHECK(mimgpu_model_set_weight(m, ws[i].name, ts[i]) == MIMGPU_OK, "bind %s: %s", ws[i].name,
              mimgpu_last_error(ctx));
    }
    mimgpu_session *s = NULL;
    CHECK(mimgpu_session_new(m, &s) == MIMGPU_OK, "session_new: %s", mimgpu_last_error(ctx));

    /* the reference side */
    const mo_llama_config oc = {L, E, F, H, HKV, D, D, V, C, 500000.0, 1e-5, 1, 1, 1, 4};
    mo_llama *ref = mo_llama_new(&oc);
    CHECK(ref != NULL, "oracle model");
    for (int i = 0; i < nw; i++)
        CHECK(mo_llama_set_weight(ref, ws[i].name, ws[i].dt, ws[i].bytes) == 0, "oracle bind %s", ws[i].name);

    int32_t prompt[P];
    int64_t pos[P];
    for (int i = 0; i < P; i++) {
        prompt[i] = (int32_t)((i * 7919 + 13) % V);
        pos[i] = i;
    }
    float got[V], want[V];
    CHECK(mimgpu_session_run(s, prompt, pos, P, got, 0) == MIMGPU_OK, "session_run: %s", mimgpu_last_error(ctx));
    CHECK(mo_llama_forward(ref, prompt, pos, P, want, 0) == 0, "oracle forward");
    CHECK(same_bits(got, want, V), "prompt logits differ from the oracle");

    int32_t tok = mo_argmax(want, V), ids[STEPS];
    CHECK(mimgpu_session_generate(s, tok, P, STEPS, ids) == MIMGPU_OK, "generate: %s", mimgpu_last_error(ctx));
    for (int i = 0; i < STEPS; i++) {
        const int64_t p1 = P + i;
        CHECK(mo_llama_forward(ref, &tok, &p1, 1, want, 0) == 0, "oracle step");
        tok = mo_argmax(want, V);
        CHECK(ids[i] == tok, "greedy id %d: %d, the oracle %d", i, ids[i], tok);
    }

    mo_llama_free(ref);
    mimgpu_session_free(s);
    mimgpu_model_free(m);
    for (int i = 0; i < nw; i++) {
        mimgpu_tensor_free(ts[i]);
        free(ws[i].bytes);
    }
}

int main(void) {
    CHECK(mimgpu_abi_version() == MIMGPU_ABI_VERSION, "ABI version %d, header %d", mimgpu_abi_version(),
          MIMGPU_ABI_VERSION);
    mimgpu_ctx *ctx = NULL;
    CHECK(mimgpu_open(0, &ctx) == MIMGPU_OK, "open device 0");
    check_matmul(ctx);
    check_model(ctx);
    mimgpu_close(ctx);
    printf("capi driver ok\n");
    return 0;
}
