// sparse.cu — Backend::sparse_attention (LightX2V video sparse attention,
// crates/lightx2v-core/src/backend.rs:309-331; the VSA geometry
// crates/lightx2v-core/src/sparse.rs; CPU reference
// crates/lightx2v-cpu/src/lib.rs:496-606):
//   1. tile the (T, H, W) token grid into 4x4x4 cubes (the host builds the
//      reference's TilePlan: slot -> token, tokens per tile);
//   2. coarse: mean-pool Q, K, V per tile, dense softmax attention over tiles;
//   3. select the top-k key tiles per query tile by the coarse scores (ties to
//      the lower tile index);
//   4. fine: attention from each token to the tokens of its tile's selected
//      tiles only;
//   5. combine: out = coarse * gate + fine.
// Steps 2-3 run per (head, query tile) in the kernels below, which also write
// the fine stage's token-level visibility bits per head; the fine attention
// itself runs on the attention kernels (attention_sm100.cu) with that mask.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include "sparse.h"

namespace lx2v {

namespace {

__device__ __forceinline__ float ldv(const void *p, int f32, int64_t i) {
    return f32 ? reinterpret_cast<const float *>(p)[i] : __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[i]);
}

// Mean of each tile's tokens, as the reference sums them (slot order,
// x / n added one at a time, n = the tile's real tokens, at least 1).
// Grid (tiles, heads), thread = channel.
__global__ void vsa_pool_kernel(VsaArgs a) {
    const int t = blockIdx.x, h = blockIdx.y;
    const int n = a.block_sizes[t];
    const float nf = (float)(n > 0 ? n : 1);
    for (int j = threadIdx.x; j < a.d; j += blockDim.x) {
        float sq = 0.0f, sk = 0.0f, sv = 0.0f;
        for (int s = 0; s < n; ++s) {
            const int64_t tok = a.slot_src[(int64_t)t * VSA_TILE + s];
            const int64_t i = ((int64_t)h * a.seq + tok) * a.d + j;
            sq += ldv(a.q, a.qkv_f32, i) / nf;
            sk += ldv(a.k, a.qkv_f32, i) / nf;
            sv += ldv(a.v, a.qkv_f32, i) / nf;
        }
        const int64_t o = ((int64_t)h * a.nt + t) * a.d + j;
        a.cq[o] = sq;
        a.ck[o] = sk;
        a.cv[o] = sv;
    }
}

// Coarse attention of query tile qi (softmax_row of cpu lib.rs:155-166 on
// the tile scores) and its top-k key tiles as a bit set. Grid (tiles, heads),
// dynamic shared memory: nt scores + 32 floats of reduction scratch.
__global__ void vsa_coarse_kernel(VsaArgs a) {
    extern __shared__ float vs_smem[];
    float *row = vs_smem;
    float *red = vs_smem + a.nt;
    const int qi = blockIdx.x, h = blockIdx.y;
    const float *cq = a.cq + ((int64_t)h * a.nt + qi) * a.d;
    const float *ck = a.ck + (int64_t)h * a.nt * a.d;
    const float *cv = a.cv + (int64_t)h * a.nt * a.d;
    for (int ki = threadIdx.x; ki < a.nt; ki += blockDim.x) {
        float s = 0.0f;
        for (int j = 0; j < a.d; ++j) s += cq[j] * ck[(int64_t)ki * a.d + j];
        row[ki] = s * a.scale;
    }
    __syncthreads();
    if (threadIdx.x == 0) {  // the reference's sequential max, exp, sum and reciprocal
        float m = -INFINITY;
        for (int i = 0; i < a.nt; ++i) m = fmaxf(m, row[i]);
        float sum = 0.0f;
        for (int i = 0; i < a.nt; ++i) {
            row[i] = expf(row[i] - m);
            sum += row[i];
        }
        red[0] = 1.0f / sum;
    }
    __syncthreads();
    const float inv = red[0];
    for (int i = threadIdx.x; i < a.nt; i += blockDim.x) row[i] *= inv;
    __syncthreads();
    float *co = a.coarse_out + ((int64_t)h * a.nt + qi) * a.d;
    for (int j = threadIdx.x; j < a.d; j += blockDim.x) {
        float acc = 0.0f;
        for (int ki = 0; ki < a.nt; ++ki) acc += row[ki] * cv[(int64_t)ki * a.d + j];
        co[j] = acc;
    }
    // top-k: tile ki is kept when fewer than topk tiles rank before it
    // (higher score, or equal score and lower index)
    uint32_t *sel = a.sel + ((int64_t)h * a.nt + qi) * a.sel_words;
    for (int w = threadIdx.x; w < a.sel_words; w += blockDim.x) sel[w] = 0u;
    __syncthreads();
    for (int ki = threadIdx.x; ki < a.nt; ki += blockDim.x) {
        const float s = row[ki];
        int rank = 0;
        for (int kj = 0; kj < a.nt && rank < a.topk; ++kj) {
            const float o = row[kj];
            rank += (o > s) || (o == s && kj < ki);
        }
        if (rank < a.topk) atomicOr(sel + (ki >> 5), 1u << (ki & 31));
    }
}

// Token-level visibility of the fine stage, per head: bit k of query q's row
// is set when key k's tile is selected for q's tile. Grid (seq, heads).
__global__ void vsa_mask_kernel(VsaArgs a) {
    const int q = blockIdx.x, h = blockIdx.y;
    const int qt = a.token_tile[q];
    const uint32_t *sel = a.sel + ((int64_t)h * a.nt + qt) * a.sel_words;
    uint32_t *row = a.bits + ((int64_t)h * a.seq + q) * a.words;
    for (int w = threadIdx.x; w < a.words; w += blockDim.x) {
        uint32_t bits = 0;
        for (int b = 0; b < 32; ++b) {
            const int k = w * 32 + b;
            if (k >= a.seq) break;
            const int kt = a.token_tile[k];
            bits |= ((sel[kt >> 5] >> (kt & 31)) & 1u) << b;
        }
        row[w] = bits;
    }
}

// out[q, h*d + j] = coarse_out[h][tile(q)][j] * gate[h][q][j] + fine[q, h*d + j], in place on fine.
__global__ void vsa_combine_kernel(VsaArgs a) {
    const int64_t total = (int64_t)a.seq * a.heads * a.d;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = i % a.d, hq = i / a.d;
        const int64_t h = hq % a.heads, q = hq / a.heads;
        const float c = a.coarse_out[(h * a.nt + a.token_tile[q]) * a.d + j];
        const float g = ldv(a.gate, a.gate_f32, (h * a.seq + q) * a.d + j);
        const float f = ldv(a.out, a.out_f32, i);
        const float o = c * g + f;
        if (a.out_f32) reinterpret_cast<float *>(a.out)[i] = o;
        else reinterpret_cast<__nv_bfloat16 *>(a.out)[i] = __float2bfloat16_rn(o);
    }
}

}  // namespace

cudaError_t vsa_select_launch(const VsaArgs &a, cudaStream_t st) {
    vsa_pool_kernel<<<dim3(a.nt, a.heads), 128, 0, st>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const size_t smem = ((size_t)a.nt + 32) * sizeof(float);
    if (smem > 48 * 1024) {
        e = cudaFuncSetAttribute(vsa_coarse_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    vsa_coarse_kernel<<<dim3(a.nt, a.heads), 256, smem, st>>>(a);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    vsa_mask_kernel<<<dim3(a.seq, a.heads), 128, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t vsa_combine_launch(const VsaArgs &a, cudaStream_t st) {
    const int64_t total = (int64_t)a.seq * a.heads * a.d;
    const int blocks = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
    vsa_combine_kernel<<<blocks, 256, 0, st>>>(a);
    return cudaGetLastError();
}

}  // namespace lx2v
