// model_kernels.h -- launchers of the device-resident llama step kernels.
#pragma once

#include <cuda.h>  // CUtensorMap (types only)

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "kernels.h"

struct mimgpu_tp;

namespace mimgpu {

// tensor parallelism (tp.cu): group size and rank (1, 0 without a group),
// the all-gather of `count` floats per rank and the 64-bit max all-reduce
int tp_size(const mimgpu_tp *tp);
int tp_rank(const mimgpu_tp *tp);
cudaError_t tp_allgather(mimgpu_tp *tp, const float *send, float *recv, size_t count, cudaStream_t st);
cudaError_t tp_allreduce_max_u64(mimgpu_tp *tp, unsigned long long *buf, cudaStream_t st, size_t count = 1);
// [N][T][W] -> rows of stride ldd, columns below wmax; and the [T][W] slab
// of columns [c0, c0 + W) of rows of stride ld
cudaError_t launch_unshard(const float *src, int N, int T, int W, float *dst, long long ldd, long long wmax,
                           cudaStream_t st);
cudaError_t launch_pack(const float *x, int T, long long ld, long long c0, int W, float *y, cudaStream_t st);

struct RopeScatterArgs {
    const float *qkv;      // [T, ldq]: q (H*D) | k (Hkv*D) | v (Hkv*D)
    long long ldq;
    const int64_t *pos;    // [T]
    const double *inv_freq;
    int T, H, Hkv, D, C, rotary, interleaved, cache_f16;
    float *qh;             // [H, T, D]
    void *kc, *vc;         // [slots][Hkv, C, D]
    const int32_t *slot;   // [T] sequence (cache) of each row, or null: every row in sequence slot0
    int slot0;
    // the session's (f32(cos), f32(sin)) of pos * inv_freq[i] computed in
    // float64, [C][rotary/2] (the same values sincos gives here), or null
    const float2 *rope_cs;
};
// elements of one sequence's cache of one layer
__host__ __device__ inline long long cache_slot_elems(int Hkv, int C, int D) { return (long long)Hkv * C * D; }

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
    float *scores;     // many-row kernel: score scratch of attn_prefill_scores_bytes, or null
    const int32_t *slot;  // [T] sequence of each row (batched decoding), or null: sequence slot0
    int slot0;
    P2P put;              // tensor parallelism, one row: outputs also into every rank's full vector (N > 1)
};

cudaError_t launch_rope_scatter(const RopeScatterArgs &a, cudaStream_t st, bool pdl);
// whether launch_attn_exact runs these arguments through the many-row kernel
// (given act.q null)
bool attn_prefill_ok(const AttnArgs2 &a);
size_t attn_prefill_scores_bytes(int T, int H, int Hkv, int C);
// Dynamic shared memory of the attention kernel: q and the scores of the
// 256/D heads of a block over the whole context, plus the key/value chunk
// ring (kAttnRing buffers of kAttnChunk keys of every kv head the block
// reads).
constexpr size_t kAttnSmemMax = 220 * 1024;
// From this many query rows (a prompt pass) with an f16 cache and D = 128,
// the rows go through the many-row kernel (same bits per row) and the
// caller quantizes the outputs separately (act.q must be null then).
constexpr int kAttnPrefillMinRows = 8;
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
// The attention of a decode step with the token's RoPE and cache write fused
// in (k_attn_decode.cu): same bits as launch_rope_scatter + launch_attn_exact.
// Rows are single tokens of distinct sequences (T == 1, or one slot per row);
// D == 128, an even group size, an f16 cache and C <= attn_decode_max_context().
// It reads pos and the cache rows below pos before its grid dependency wait:
// the caller's forward must start with a kernel that waits for the previous
// forward before it lets its dependents launch (embedding_kernel does).
struct AttnDecodeArgs {
    CUtensorMap kmap[2];   // the layer's key cache [slots * Hkv][C][D] f16: boxes [64][256][1], [64][128][1], 128-byte swizzle
    AttnArgs2 at;          // qh unused
    const float *qkv;      // [T, ldq]: q (H*D) | k (Hkv*D) | v (Hkv*D), before RoPE
    long long ldq;
    const float2 *rope_cs; // [C][rotary/2]: f32(cos), f32(sin) of pos * inv_freq[i] (float64)
    int rotary, interleaved;
};
int attn_decode_max_context();
// The key-cache maps of one layer for launch_attn_decode, one per chunk size
// (false: no driver encoder).
bool attn_decode_kmap(const void *kc, int slots, int Hkv, int C, CUtensorMap out[2]);
bool attn_decode_ok(const AttnArgs2 &a);
cudaError_t launch_attn_decode(const AttnDecodeArgs &a, cudaStream_t st, bool pdl);
// wait / keys: tensor parallelism, the ranks' keys arrive in keys[0..N)
cudaError_t launch_advance(unsigned long long *key, int32_t *tok, int64_t *pos, int32_t *ids, int *step,
                           cudaStream_t st, bool pdl, const P2P *wait = nullptr,
                           const unsigned long long *keys = nullptr, int rows = 1);

}  // namespace mimgpu
