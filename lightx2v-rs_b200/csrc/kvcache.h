// kvcache.h — device data movement of the KV cache (kvcache.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace lx2v {

// dst[h][dst_row0 + r][:] = src[h][src_row0 + r][:] for r < rows (d values a
// row, head strides src_hs / dst_hs rows), bf16 or f32 on either side.
cudaError_t kv_copy_rows_launch(const void *src, int src_f32, int64_t src_hs, int64_t src_row0, void *dst,
                                int dst_f32, int64_t dst_hs, int64_t dst_row0, int64_t rows, int d, int heads,
                                cudaStream_t st);
// rows [ema_row0, +rows) <- (1 - alpha) * themselves + alpha * rows [src_row0, +rows), every head.
cudaError_t kv_ema_launch(__nv_bfloat16 *data, int64_t hs, int64_t ema_row0, int64_t src_row0, int64_t rows, int d,
                          int heads, float alpha, cudaStream_t st);

}  // namespace lx2v
