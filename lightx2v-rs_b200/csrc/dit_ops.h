// dit_ops.h — the DiT block's row-wise / elementwise ops (dit_ops.cu).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace lx2v {

// layer_norm / residual_norm: rows of width dim; kind 0 = affine (w, b),
// 1 = modulated by the mods table's rows `scale` and `shift`.
struct NormArgs {
    const void *x; int x_f32;
    void *out; int out_f32;
    int64_t rows;
    int dim;
    int kind;
    const void *w; int w_f32;
    const void *b; int b_f32;
    const void *mods; int mods_f32;
    int scale, shift;
    float eps;
};

struct HeadSplitArgs {
    const void *src; int src_f32;
    int64_t rows, src_stride, col_off;
    int heads, head_dim;
    const void *rms_w; int w_f32;     // null: no RMS norm
    const float *sumsq;               // null: the RMS statistic is this row's own; else [parts][rows] sums of
    int sumsq_parts;                  //   squares (the parts added; one per tensor-parallel rank)
    int64_t sumsq_stride;             //   elements between parts
    int rms_dim;                      //   squares over rms_dim values (all heads, summed across ranks)
    const void *cos, *sin; int cs_f32; // null: no RoPE; [rows][head_dim / 2]
    float eps;
    void *out; int out_f32;           // [heads][rows][head_dim]
};

bool row_op_supported(int dim);  // rows of at most 4096 values
cudaError_t layer_norm_launch(const NormArgs &a, cudaStream_t st);
cudaError_t residual_norm_launch(const NormArgs &a, void *h, int h_f32, const void *res, int res_f32, int gate,
                                 cudaStream_t st);
cudaError_t head_split_launch(const HeadSplitArgs &a, cudaStream_t st);
// to_tokens 1: latent [c, t, h, w] -> tokens [t*(h/p)*(w/p), c*p*p]; 0: back.
// out[r] = sum of src[r * stride + col_off + j]^2 for j < width (f32).
cudaError_t row_sumsq_launch(const void *src, int src_f32, int64_t rows, int64_t stride, int64_t col_off, int width,
                             float *out, cudaStream_t st);
cudaError_t patchify_launch(const void *src, int src_f32, void *dst, int dst_f32, int c, int t, int h, int w, int p,
                            int to_tokens, cudaStream_t st);
cudaError_t dmd_step_launch(void *x, int x_f32, const void *v, int v_f32, const void *noise, int n_f32, float sigma_t,
                            float sigma_next, int64_t n, cudaStream_t st);

}  // namespace lx2v
