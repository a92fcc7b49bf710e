// gemm.h — parameters and launchers of the linear kernels.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <atomic>
#include <cstdint>

namespace lx2v {

// A launcher's one-time set-up (the shared-memory opt-in, which is per
// device, and the occupancy it yields), cached per device: 0 until the first
// launch on that device. A device index past the table gets no cache (the
// set-up runs every launch).
constexpr int LX2V_MAX_DEVICES = 64;
inline std::atomic<int> *device_slot(std::atomic<int> (&cache)[LX2V_MAX_DEVICES]) {
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= LX2V_MAX_DEVICES) return nullptr;
    return &cache[d];
}

// Everything one linear launch needs; passed by value as a __grid_constant__.
struct alignas(64) GemmParams {
    CUtensorMap tmap_x;  // x: bf16 [x_row + M, K], box {64, BT}, 128-byte swizzle
    CUtensorMap tmap_w;  // weight codes [N rows], box {one 64-wide k-block, 128 rows}
    CUtensorMap tmap_s;  // scale words [G][N] (4 bytes each), box {128 rows, sgrp groups}
    CUtensorMap tmap_f;  // FP8 block flags [ceil(K/32)][N] bytes, box {128 rows, 2}
    CUtensorMap tmap_y;  // two-pass kernel with tma_y: y [y_row + M][N] (bf16 or f32), box {32, 32}
    void *y;                  // output (or h for the gated residual)
    const uint8_t *codes;     // weight codes in the reference layout (dequant.cuh)
    const float *scales_t;    // Q8/FP8 scales, [G][N]
    const uint32_t *sz_t;     // Q4 (scale, zero) half2 words, [G][N]
    const void *bias;         // [N] or null
    const void *gate;         // [N] (mods + gate * N) or null
    int *err;                 // error word (ptx.cuh error codes)
    uint64_t wait_limit_ns;   // bounded-wait limit
    int M, N, K, group;
    int x_row, y_row;
    int act;                  // 0 none, 1 GELU-tanh
    int out_f32;              // y element type: 1 f32, 0 bf16
    int reduce;               // 1: reduce-add into y (gated residual)
    int bias_f32, gate_f32;   // element types of bias / gate
    int sgrp;                 // scale groups per k-block box (1, 2 or 4)
    int gshift;               // log2(group) when group < 64, else 6
    // Stream-K (pair kernels): when streamk != 0 the tiles' k-blocks are split
    // into equal contiguous ranges, one per CTA pair. A pair whose range
    // starts inside a tile writes that partial tile's f32 accumulator to
    // partials[(pair * 2 + rank) * 128 * bt ...] and publishes `epoch` in
    // flags[pair * 2 + rank] (two-pass kernel: one flag per epilogue warp,
    // flags[(pair * 2 + rank) * 8 + warp]); the pair holding the tile's first
    // k-block adds those partials in its epilogue.
    int streamk;
    int epoch;
    int kgroup;               // pair kernel: k-blocks per MMA group (1, or 2 when K % 128 == 0)
    int tma_y;                // two-pass kernel: y written by TMA tensor stores (reduce-add for f32 residuals)
    // Two-pass kernel, whole-tile mode with a reduce-add epilogue and no
    // activation: every tile's k-blocks split into `ksplit` ranges, each a
    // work item of its own that reduce-adds gate * partial into y (the bias
    // with the first range only). 0 or 1: whole tiles.
    int ksplit;
    float *partials;
    int *flags;
};

// Tensor-core (tcgen05) dequant GEMM. `bt` = token tile (128, 192 or 256).
cudaError_t gemm_dq_launch(int fmt, int bt, const GemmParams &p, int num_sms, cudaStream_t st);
int gemm_dq_token_tile(int M, int N, int K, int units, int feat_tile);
// The same GEMM on CTA pairs (cta_group::2): pair tile = 256 features x bt
// tokens; tmap_x's box must be {64, bt/2}.
cudaError_t gemm_pair_launch(int fmt, int bt, const GemmParams &p, int num_sms, cudaStream_t st);
// Second pass of the two-pass linear (gemm_ss_sm100.cu): tmap_w maps a bf16
// [N][K] weight (box {64, 128}, 128-byte swizzle), tmap_x has box {64, bt/2}.
cudaError_t gemm_ss_pair_launch(int bt, const GemmParams &p, int num_sms, cudaStream_t st);
int gemm_ss_token_tile(int M, int N, int K, int pairs);
int gemm_ss_ksplit(int M, int N, int K, int bt, int pairs);

// Small-M path and the generic CUDA-core path (kernels.cu); they take plain
// pointers instead of tensor maps.
struct LinearArgs {
    int fmt;
    const uint8_t *codes;
    const float *scales_t;
    const uint32_t *sz_t;
    const uint8_t *flags;     // FP8 block flags, [ceil(K/32)][N]
    int M, N, K, group;
    const void *x; int x_f32; int64_t x_row;
    void *y; int y_f32; int64_t y_row;
    const void *bias; int bias_f32;
    const void *gate; int gate_f32;   // non-null: y += gate * act(...)
    int act;
    int *err;                 // error word for bounded waits (gemv_q4.cu), may be null
    uint64_t wait_limit_ns;
};
cudaError_t linear_simt_launch(const LinearArgs &a, cudaStream_t st);
// Few-token (M <= 16) bandwidth-bound kernel (gemv.cu). Split-K partials go
// to `partials` (gemv_workspace_floats(N, K, num_sms) floats) and `arrivals`
// (ceil(N / 64) ints, zero before the first launch; the kernel leaves them
// zero).
bool gemv_supported(const LinearArgs &a);
size_t gemv_workspace_floats(int N, int K, int num_sms);
cudaError_t linear_gemv_launch(const LinearArgs &a, int num_sms, cudaStream_t st, float *partials, int *arrivals,
                               size_t ws_floats);
// Few-token Q4 kernel with the group affine applied after the products
// (gemv_q4.cu): K and the group multiples of 64; no workspace (partials meet
// in the cluster's shared memory). linear_gemv_launch takes it for Q4 when
// gemv_q4_supported.
bool gemv_q4_supported(const LinearArgs &a, int num_sms);
cudaError_t gemv_q4_launch(const LinearArgs &a, int num_sms, cudaStream_t st);

// Elementwise helpers (kernels.cu).
cudaError_t convert_launch(const void *src, int src_f32, void *dst, int dst_f32, size_t n,
                           cudaStream_t st);
cudaError_t gate_residual_launch(void *h, int h_f32, const void *a, int a_f32, const void *gate,
                                 int gate_f32, size_t rows, size_t dim, cudaStream_t st);
// First pass of the two-pass linear: the weight decoded to bf16, [N][K].
cudaError_t dequant_bf16_launch(int fmt, const uint8_t *codes, const float *scales_t, const uint32_t *sz_t,
                                const uint8_t *flags, int N, int K, int group, __nv_bfloat16 *out,
                                cudaStream_t st);
cudaError_t dequant_f32_launch(int fmt, const uint8_t *codes, const float *scales_t,
                               const uint32_t *sz_t, const uint8_t *flags, int N, int K, int group,
                               float *out, cudaStream_t st);

}  // namespace lx2v
