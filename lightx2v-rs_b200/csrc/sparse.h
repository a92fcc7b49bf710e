// sparse.h — video sparse attention (sparse.cu).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace lx2v {

constexpr int VSA_TILE = 64;  // 4 x 4 x 4 tokens per tile (crates/lightx2v-core/src/sparse.rs:21-22)

struct VsaArgs {
    int heads, seq, d, nt, topk;
    float scale;
    const void *q, *k, *v;           // [heads][seq][d]
    int qkv_f32;
    const void *gate; int gate_f32;  // [heads][seq][d]
    void *out; int out_f32;          // [seq][heads * d]: the fine attention, then the combined result
    const uint32_t *slot_src;        // [nt * 64] source token of each slot (0xFFFFFFFF padding)
    const int *block_sizes;          // [nt] real tokens per tile
    const int *token_tile;           // [seq]
    float *cq, *ck, *cv;             // [heads][nt][d] tile means
    float *coarse_out;               // [heads][nt][d]
    uint32_t *sel;                   // [heads][nt][sel_words] selected key tiles per query tile
    int sel_words;
    uint32_t *bits;                  // [heads][seq][words] fine-stage visibility
    int words;
};

// Pooling, coarse attention, top-k selection and the fine-stage mask.
cudaError_t vsa_select_launch(const VsaArgs &a, cudaStream_t st);
// out = coarse * gate + out (the fine attention).
cudaError_t vsa_combine_launch(const VsaArgs &a, cudaStream_t st);

}  // namespace lx2v
