// step.h -- the one-token decode step of the llama graph (importer/llama.go:
// 400-534 of gsoultan/mimir-model) as ONE persistent kernel (k_step.cu).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "kernels.h"

namespace mimgpu {

// One decoder layer's weights (byte-exact block rows) and cache.
struct StepLayer {
    const uint8_t *w[7];  // attn_q, attn_k, attn_v, attn_output, ffn_gate, ffn_up, ffn_down
    int dt[7];            // Q4_K or Q6_K
    const float *attn_norm, *ffn_norm;
    void *kc, *vc;        // f16 [Hkv][C][D] (sequence 0 of the session)
};

struct StepParams {
    const StepLayer *layers;  // device array [L]
    int L, E, F, H, Hkv, D, V, C, rotary;
    float eps, scale;
    const uint8_t *embd;
    int embd_dt;
    const uint8_t *head;
    int head_dt;
    const float *out_norm;
    const float2 *rope_cs;    // [C][rotary/2]: f32(cos), f32(sin) of pos * inv_freq[i]
    const int32_t *tok;       // [1] token of this step
    const int64_t *pos;       // [1] its position
    float *x;                 // [E] residual stream
    float *qh;                // [H][D] query heads after RoPE
    float *att;               // [E] attention output
    float *a;                 // [F] SwiGLU output
    float *logits;            // [V]
    ActQ8 actE, actF;         // 8-bit blocks of att and a
    unsigned long long *amax; // greedy key (folded with atomicMax), or null
    unsigned *sync;           // grid counters, step_sync_words(L, F) words, zero at session start
    unsigned *epoch;          // [0] steps completed, [1] CTA exits; zero at session start
    unsigned *status;         // device status word (wait limit in ns at status + 2)
    unsigned long long *trace;  // phase timeline [G][step_trace_words(L)] (%globaltimer ns), or null
};

// Timeline slots of one CTA: [0] start, [1] end, then 16 per job (4 per
// layer + the head): 0 activation ready, 1 activation in shared memory, 2
// consumer stages done, 3 attention unit done, 4 chain warps done, 5 first
// stage issued, 6 last stage issued; for the o job of an attention CTA also
// 8 q|k|v rows of every CTA written, 9 first key stage landed, 10 scores done,
// 11 softmax sums done, 12 weighted sums done.
// After the CTAs' slots: CTA 0's stage log, kStageLog entries of 4 words
// (consumer warp 0 after the stage landed, after its record stage was free,
// when its records were written; chain warp done with the record stage).
constexpr int kStageLog = 1024;
__host__ __device__ inline size_t step_trace_cta_words(int L) { return 2 + 16 * (size_t)(4 * L + 1); }
__host__ __device__ inline size_t step_trace_words_total(int G, int L) {
    return (size_t)G * step_trace_cta_words(L) + 4 * (size_t)kStageLog;
}

// Whether a model of these dimensions runs through the step kernel (else the
// kernel-per-op path): Q4_K / Q6_K matrices, E a multiple of 256 up to 8192,
// F up to 32768, head size 128 with 2, 4, 8 ... query heads per kv head, an f16 cache
// whose attention scratch fits shared memory, interleaved RoPE.
bool step_ok(int E, int F, int H, int Hkv, int D, int C, int rotary, int interleaved, int cache_f16);
size_t step_sync_words(int L, int F);
cudaError_t step_prepare();
cudaError_t launch_step(const StepParams &p, cudaStream_t st);
// cs[pos][i] = (f32(cos(pos * inv_freq[i])), f32(sin(...))) for pos < C, i < half
cudaError_t launch_rope_table(const double *inv_freq, int C, int half, float2 *cs, cudaStream_t st);

}  // namespace mimgpu
