// kvcache.cu — data movement of the per-layer KV cache (Backend::kv_cache_*,
// crates/lightx2v-core/src/backend.rs:334-390; CPU reference
// crates/lightx2v-cpu/src/lib.rs:607-806). The cache keeps K and V as
// [heads][capacity rows][head_dim] bf16, so that one head's keys are one
// contiguous [rows][head_dim] matrix the attention kernel reads by TMA; the
// slot bookkeeping (temporal indices, slot kinds) lives on the host.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include "kvcache.h"

namespace lx2v {

namespace {

__device__ __forceinline__ float ld_any(const void *p, int f32, int64_t i) {
    return f32 ? reinterpret_cast<const float *>(p)[i] : __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[i]);
}
__device__ __forceinline__ void st_any(void *p, int f32, int64_t i, float v) {
    if (f32) reinterpret_cast<float *>(p)[i] = v;
    else reinterpret_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v);
}

// dst[h][dst_row0 + r][c] = src[h][src_row0 + r][c] for r < rows, c < d,
// converting between element types; head strides in rows.
__global__ void kv_copy_rows_kernel(const void *src, int src_f32, int64_t src_hs, int64_t src_row0, void *dst,
                                    int dst_f32, int64_t dst_hs, int64_t dst_row0, int64_t rows, int d, int heads) {
    const int64_t per_head = rows * d;
    const int64_t total = per_head * heads;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t h = i / per_head, e = i % per_head;
        const int64_t r = e / d, c = e % d;
        const float v = ld_any(src, src_f32, (h * src_hs + src_row0 + r) * d + c);
        st_any(dst, dst_f32, (h * dst_hs + dst_row0 + r) * d + c, v);
    }
}

// The same copy between equal element types, 16 bytes a thread: rows of
// row_vec uint4 per head (head strides in rows).
__global__ void kv_copy_rows_vec_kernel(const uint4 *src, int64_t src_hs, int64_t src_row0, uint4 *dst,
                                        int64_t dst_hs, int64_t dst_row0, int64_t rows, int row_vec, int heads) {
    const int64_t per_head = rows * row_vec;
    const int64_t total = per_head * heads;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t h = i / per_head, e = i % per_head;
        dst[(h * dst_hs + dst_row0) * row_vec + e] = src[(h * src_hs + src_row0) * row_vec + e];
    }
}

// ema rows <- (1 - alpha) * ema + alpha * frame rows (memrope.rs ema_update),
// in f32 on the stored bf16 values.
__global__ void kv_ema_kernel(__nv_bfloat16 *data, int64_t hs, int64_t ema_row0, int64_t src_row0, int64_t rows,
                              int d, int heads, float alpha) {
    const int64_t per_head = rows * d;
    const int64_t total = per_head * heads;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t h = i / per_head, e = i % per_head;
        const int64_t base = h * hs * d;
        const float em = __bfloat162float(data[base + ema_row0 * d + e]);
        const float f = __bfloat162float(data[base + src_row0 * d + e]);
        data[base + ema_row0 * d + e] = __float2bfloat16_rn((1.0f - alpha) * em + alpha * f);
    }
}

int grid_for(int64_t n) {
    int64_t b = (n + 255) / 256;
    return (int)(b < 1 ? 1 : (b > 65535 * 4 ? 65535 * 4 : b));
}

}  // namespace

cudaError_t kv_copy_rows_launch(const void *src, int src_f32, int64_t src_hs, int64_t src_row0, void *dst,
                                int dst_f32, int64_t dst_hs, int64_t dst_row0, int64_t rows, int d, int heads,
                                cudaStream_t st) {
    if (rows <= 0 || heads <= 0) return cudaSuccess;
    if (src_f32 == dst_f32) {
        const size_t es = src_f32 ? 4 : 2;
        if (((size_t)d * es) % 16 == 0 && reinterpret_cast<uintptr_t>(src) % 16 == 0 &&
            reinterpret_cast<uintptr_t>(dst) % 16 == 0) {
            // same element type, 16-byte rows: a vector copy on the SMs (the
            // strided cudaMemcpy2DAsync ran at ~1.5 TB/s on the chunk's K / V)
            const int row_vec = (int)((size_t)d * es / 16);
            const int64_t n = rows * row_vec * heads;
            const int64_t b = (n + 255) / 256;
            kv_copy_rows_vec_kernel<<<(int)(b < 148 * 16 ? b : 148 * 16), 256, 0, st>>>(
                reinterpret_cast<const uint4 *>(src), src_hs, src_row0, reinterpret_cast<uint4 *>(dst), dst_hs,
                dst_row0, rows, row_vec, heads);
            return cudaGetLastError();
        }
        // same element type otherwise: one strided copy, a row block per head
        return cudaMemcpy2DAsync((char *)dst + (size_t)dst_row0 * d * es, (size_t)dst_hs * d * es,
                                 (const char *)src + (size_t)src_row0 * d * es, (size_t)src_hs * d * es,
                                 (size_t)rows * d * es, (size_t)heads, cudaMemcpyDeviceToDevice, st);
    }
    kv_copy_rows_kernel<<<grid_for(rows * d * heads), 256, 0, st>>>(src, src_f32, src_hs, src_row0, dst, dst_f32,
                                                                    dst_hs, dst_row0, rows, d, heads);
    return cudaGetLastError();
}

cudaError_t kv_ema_launch(__nv_bfloat16 *data, int64_t hs, int64_t ema_row0, int64_t src_row0, int64_t rows, int d,
                          int heads, float alpha, cudaStream_t st) {
    if (rows <= 0 || heads <= 0) return cudaSuccess;
    kv_ema_kernel<<<grid_for(rows * d * heads), 256, 0, st>>>(data, hs, ema_row0, src_row0, rows, d, heads, alpha);
    return cudaGetLastError();
}

}  // namespace lx2v
