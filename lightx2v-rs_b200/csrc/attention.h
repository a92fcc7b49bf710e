// attention.h — parameters and launchers of the attention kernels
// (attention_sm100.cu).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace lx2v {

enum : int { ATT_MASK_NONE = 0, ATT_MASK_BITS = 1, ATT_MASK_TEMPORAL = 2 };

// Tensor-core kernel: head_dim 128, bf16 Q/K/V.
struct alignas(64) AttnParams {
    CUtensorMap tmap_q;   // Q bf16 [heads * q_rows][128], box {64, 128}, 128-byte swizzle
    CUtensorMap tmap_k;   // K bf16 [heads * k_rows][128], box {64, 128}, 128-byte swizzle
    CUtensorMap tmap_v;   // V bf16 as stored, 3-D {128, sk, heads} (head stride k_rows rows), box {64, 128, 1},
                          // 128-byte swizzle: keys >= sk of a head arrive as zeros
    void *out;            // [sq][heads * 128], bf16 or f32
    int out_f32;
    int heads, sq, sk;
    int q_rows, k_rows;   // rows per head of the Q and K tensors (>= sq, >= sk)
    float scale_log2;     // log2(e) / sqrt(128)
    int mask_mode;        // ATT_MASK_*
    const uint32_t *mask_bits;  // [sq][mask_words] (bit k % 32 of word k / 32: key k visible)
    int mask_words;
    int64_t mask_head_stride;   // words between the heads' masks (0: one mask for all heads)
    const int *tq;        // [sq] temporal index of each query (mask_mode TEMPORAL)
    const int *tk;        // [sk] temporal index of each key
    const int2 *tk_range; // [ceil(sk / 128)] (min, max) tk of each key block
    const int2 *tq_range; // [ceil(sq / 128)] (min, max) tq of each query tile
    const int *tile_order;  // [ceil(sq / 128)] query tiles, most key blocks first (or null: in order)
    int *err;
    uint64_t wait_limit_ns;
};

// Generic kernel: any head_dim up to 256, f32 or bf16 buffers.
struct AttnSimtParams {
    const void *q, *k, *v;
    int qkv_f32;
    void *out;
    int out_f32;
    int heads, sq, sk, d;
    int q_rows, k_rows;
    int mask_mode;
    const uint32_t *mask_bits;
    int mask_words;
    int64_t mask_head_stride;
    const int *tq, *tk;
};

cudaError_t attention_tc_launch(const AttnParams &p, cudaStream_t st);
cudaError_t attention_simt_launch(const AttnSimtParams &p, cudaStream_t st);
}  // namespace lx2v
