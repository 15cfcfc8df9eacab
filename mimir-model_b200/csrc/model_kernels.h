// model_kernels.h -- launchers of the device-resident llama step kernels.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "kernels.h"

namespace mimgpu {

struct RopeScatterArgs {
    const float *qkv;      // [T, ldq]: q (H*D) | k (Hkv*D) | v (Hkv*D)
    long long ldq;
    const int64_t *pos;    // [T]
    const double *inv_freq;
    int T, H, Hkv, D, C, rotary, interleaved, cache_f16;
    float *qh;             // [H, T, D]
    void *kc, *vc;         // [Hkv, C, D]
};

// Attention of the model step: q heads [H, T, D] (after RoPE) over the cache
// [Hkv, C, D], keys [0, pos[t]] for query row t; out [T, H*D] and, when
// act.q is set, its 8-bit blocks.
struct AttnArgs2 {
    const float *qh;
    const void *kc, *vc;
    const int64_t *pos;
    int T, H, Hkv, D, C, cache_f16;
    float scale;
    float *out;
    ActQ8 act;
    unsigned *status;  // device status word (bounded waits record timeouts here)
};

cudaError_t launch_rope_scatter(const RopeScatterArgs &a, cudaStream_t st, bool pdl);
// Dynamic shared memory of the attention kernel: q and the scores of the
// 256/D heads of a block over the whole context, plus the key/value chunk
// ring (kAttnRing buffers of kAttnChunk keys of every kv head the block
// reads).
constexpr size_t kAttnSmemMax = 220 * 1024;
constexpr int kAttnChunk = 64;
constexpr int kAttnRing = 4;
inline int attn_kv_per_block(int H, int Hkv, int D) {
    const int HPB = 256 / D, G = H / Hkv;
    return G >= HPB ? 1 : HPB / G + 1;  // blocks may straddle kv heads when G < HPB
}
inline size_t attn_exact_smem(int H, int Hkv, int D, int C, int f16) {
    const size_t chunk = (size_t)attn_kv_per_block(H, Hkv, D) * kAttnChunk * D * (f16 ? 2 : 4);
    return 1024 + sizeof(float) * (256 + (size_t)(256 / D) * C) + (size_t)kAttnRing * chunk;
}
cudaError_t launch_attn_exact(const AttnArgs2 &a, cudaStream_t st, bool pdl);
cudaError_t launch_advance(unsigned long long *key, const float *logits, int32_t *tok, int64_t *pos, int32_t *ids,
                           int *step, cudaStream_t st, bool pdl);

}  // namespace mimgpu
