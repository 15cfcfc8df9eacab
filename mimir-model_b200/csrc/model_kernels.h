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

struct AttnSplitArgs {
    const float *qh;       // [H, T, D]
    const void *kc, *vc;   // [Hkv, C, D]
    const int64_t *pos;    // [T]
    int T, H, Hkv, D, C, cache_f16;
    int chunk, S;          // keys per split (64), splits
    float scale;
    float *po;             // [T, H, S, D]
    float *pml;            // [T, H, S, 2]
};

struct AttnCombineArgs {
    const float *po, *pml;
    const int64_t *pos;
    int T, H, D, S, chunk;
    float *out;            // [T, H*D]
    ActQ8 act;             // q null: no quantization
};

cudaError_t launch_rope_scatter(const RopeScatterArgs &a, cudaStream_t st, bool pdl);
size_t attn_split_smem(int G, int D, int f16);
cudaError_t launch_attn_split(const AttnSplitArgs &a, cudaStream_t st, bool pdl);
cudaError_t launch_attn_combine(const AttnCombineArgs &a, cudaStream_t st, bool pdl);
cudaError_t launch_advance(const int *argmax, int32_t *tok, int64_t *pos, int32_t *ids, int *step, cudaStream_t st,
                           bool pdl);

}  // namespace mimgpu
