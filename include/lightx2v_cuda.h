/*
 * lightx2v_cuda.h — C ABI of the B200 (sm_100a) backend for lightx2v-rs: the
 * quantized linear path, and the other ops of the DiT chunk step around it
 * (attention, KV cache / MemRoPE, norms, head_split, patchify, dmd_step).
 *
 * The entry points are what a `lightx2v-cuda` crate's `impl Backend for
 * CudaBackend` binds (crates/lightx2v-core/src/backend.rs:145-446). Each
 * declaration names the trait method or reference function it serves.
 *
 * Conventions
 *   - Every call returns lx2v_status (0 = LX2V_OK). On failure the message is
 *     available from lx2v_last_error(ctx) until the next call on that ctx.
 *   - Handles are opaque and owned by the library; *_free releases them.
 *   - Host arrays passed in are copied during the call and never retained.
 *   - A context owns one CUDA stream on one device. Calls on a context are
 *     ordered on that stream. Use a context from one thread at a time; it may
 *     be moved between threads (the reference moves its backend into the
 *     serve engine thread, crates/lightx2v-cli/src/serve.rs:592-612).
 *   - Activation buffers hold bf16 or f32 elements. The trait's own buffers are
 *     bf16 on CUDA (backend.rs:9-11); f32 is offered for outputs and for the
 *     residual stream. Host data crosses the boundary as f32 in both cases.
 *   - Nothing here falls back to the CPU. A missing or unusable device is an
 *     error (LX2V_ERR_NO_DEVICE), which the Rust side maps to
 *     `CudaBackend::try_new() -> None`, like WgpuBackend::try_new
 *     (crates/lightx2v-wgpu/src/lib.rs:285-290).
 */
#ifndef LIGHTX2V_CUDA_H
#define LIGHTX2V_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define LX2V_API __attribute__((visibility("default")))
#else
#define LX2V_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef int lx2v_status;
enum {
    LX2V_OK = 0,
    LX2V_ERR_INVALID = 1,     /* bad handle, shape, offset or length */
    LX2V_ERR_CUDA = 2,        /* a CUDA runtime/driver call failed */
    LX2V_ERR_OOM = 3,         /* device allocation failed */
    LX2V_ERR_UNSUPPORTED = 4, /* valid request this build cannot run */
    LX2V_ERR_NO_DEVICE = 5,   /* no usable sm_100 device */
    LX2V_ERR_DEVICE = 6       /* a kernel reported an error (bounded wait expired) */
};

/* Epilogue activation of linear, backend.rs:38-43. */
enum { LX2V_ACT_NONE = 0, LX2V_ACT_GELU_TANH = 1 };

/* Element type of an activation buffer. */
enum { LX2V_BF16 = 0, LX2V_F32 = 1 };

/* Storage format of a weight matrix (quant.rs:27-43). */
enum { LX2V_W_BF16 = 0, LX2V_W_Q8 = 1, LX2V_W_Q4 = 2, LX2V_W_FP8 = 3, LX2V_W_NVFP4 = 4 };

typedef struct lx2v_ctx lx2v_ctx;
typedef struct lx2v_buf lx2v_buf;
typedef struct lx2v_weight lx2v_weight;

/* ---- context ------------------------------------------------------------ */
/* Create a context on CUDA device `device` (backend construction; the
 * reference's try_new, crates/lightx2v-wgpu/src/lib.rs:285-290). */
LX2V_API lx2v_status lx2v_init(int device, lx2v_ctx **out);
LX2V_API void lx2v_free_ctx(lx2v_ctx *ctx);
/* Message of the last failed call on ctx ("" if none). Valid until the next
 * call on ctx. NULL ctx returns the message of the last failed lx2v_init. */
LX2V_API const char *lx2v_last_error(const lx2v_ctx *ctx);
/* Backend::name, backend.rs:158. Writes a NUL-terminated name. */
LX2V_API lx2v_status lx2v_name(lx2v_ctx *ctx, char *buf, size_t cap);
/* Backend::sync, backend.rs:190: wait for queued work; also reports a kernel
 * error (LX2V_ERR_DEVICE) raised since the last sync. */
LX2V_API lx2v_status lx2v_sync(lx2v_ctx *ctx);
/* The context's CUDA stream (a cudaStream_t), for callers that order their
 * own work with the library's. */
LX2V_API void *lx2v_stream(lx2v_ctx *ctx);

/* ---- buffers (backend.rs:160-177) ---------------------------------------- */
/* Backend::alloc: `len` zero-filled elements of `dtype`. */
LX2V_API lx2v_status lx2v_buf_alloc(lx2v_ctx *ctx, size_t len, int dtype, lx2v_buf **out);
/* Backend::upload: a new buffer holding `data` converted to `dtype`. */
LX2V_API lx2v_status lx2v_buf_upload_f32(lx2v_ctx *ctx, const float *data, size_t len, int dtype,
                                lx2v_buf **out);
/* Backend::write: overwrite the first `len` elements. Calls queued after it
 * see the new contents. The copy itself runs on a second stream of the
 * context and starts as soon as the last queued operation that used `buf`
 * is done, so it overlaps kernels queued before it that do not touch `buf`.
 * From pageable host memory `data` may be reused when the call returns; from
 * page-locked memory the copy is asynchronous: keep `data` unchanged until
 * the next lx2v_sync or blocking call. */
LX2V_API lx2v_status lx2v_buf_write_f32(lx2v_ctx *ctx, lx2v_buf *buf, const float *data, size_t len);
/* Backend::download: blocking read of the first `len` elements as f32. */
LX2V_API lx2v_status lx2v_buf_download_f32(lx2v_ctx *ctx, const lx2v_buf *buf, float *out, size_t len);
/* No counterpart in the reference (its download always blocks): the same read
 * queued on the context's stream without waiting for it. `out` holds the data
 * after the next lx2v_sync (or blocking call); with page-locked `out` the
 * copy overlaps host -> device writes queued later, which is how a caller
 * pipelines consecutive steps. */
LX2V_API lx2v_status lx2v_buf_download_f32_async(lx2v_ctx *ctx, const lx2v_buf *buf, float *out, size_t len);
/* Backend::buf_len. */
LX2V_API lx2v_status lx2v_buf_len(lx2v_ctx *ctx, const lx2v_buf *buf, size_t *len);
/* Element type and device address of a buffer (for tests and benchmarks). */
LX2V_API lx2v_status lx2v_buf_info(lx2v_ctx *ctx, const lx2v_buf *buf, int *dtype, void **dev_ptr);
/* Backend::copy: dst[dst_off..][..len] = src[src_off..][..len] (converting
 * between dtypes when they differ). */
LX2V_API lx2v_status lx2v_buf_copy(lx2v_ctx *ctx, const lx2v_buf *src, size_t src_off, lx2v_buf *dst,
                          size_t dst_off, size_t len);
LX2V_API void lx2v_buf_free(lx2v_ctx *ctx, lx2v_buf *buf);

/* ---- weights (backend.rs:178-188) ---------------------------------------- */
/* Backend::weight: a [rows, cols] f32 matrix stored as bf16 (the CUDA
 * backend's native precision, quant.rs:28-29). */
LX2V_API lx2v_status lx2v_weight_f32(lx2v_ctx *ctx, const float *data, size_t rows, size_t cols,
                            lx2v_weight **out);
/* Backend::weight_q8 for Q8 (quant.rs:144-205): codes i8 [rows*cols]
 * row-major, scales f32 [rows, cols/group]. */
LX2V_API lx2v_status lx2v_weight_q8(lx2v_ctx *ctx, const int8_t *q, const float *scales, size_t rows,
                           size_t cols, size_t group, lx2v_weight **out);
/* Backend::weight_q4 for Q4 (quant.rs:212-356): `packed` is Q4::packed()
 * ((rows*cols+1)/2 bytes, element 2i in the low nibble, quant.rs:306-311);
 * scales / zeros f32 [rows*cols/group], each exactly an f16 value as
 * Q4::quantize stores them (quant.rs:280-281). A non-f16 value is rejected. */
LX2V_API lx2v_status lx2v_weight_q4(lx2v_ctx *ctx, const uint8_t *packed, const float *scales,
                           const float *zeros, size_t rows, size_t cols, size_t group,
                           lx2v_weight **out);
/* Backend::weight_fp8 for Fp8E4M3 (quant.rs:365-460): e4m3 code bytes
 * [rows*cols] and scales f32 [rows*cols/group]. Codes decode through the
 * reference's own e4m3_to_f32 (quant.rs:409-420), not hardware e4m3. */
LX2V_API lx2v_status lx2v_weight_fp8(lx2v_ctx *ctx, const uint8_t *q, const float *scales, size_t rows,
                            size_t cols, size_t group, lx2v_weight **out);
/* NVFP4 micro-block weight (no counterpart in the reference, whose design
 * names it as the next quantisation, docs/design.md:137-145): fp4 e2m1 codes
 * packed two per byte like Q4 (element 2i in the low nibble), one e4m3 scale
 * byte per 16 consecutive values of a row [rows * cols / 16] and one f32
 * global scale. w = e2m1(code) * (e4m3(block scale) * global scale), the
 * bracket rounded to f32 once (OCP e4m3). cols a multiple of 32. Linear runs
 * it through the two-pass kernel (bf16 decode, then the CTA-pair GEMM) or
 * the generic kernel; lx2v_weight_dequant_f32 gives the exact f32 values. */
LX2V_API lx2v_status lx2v_weight_nvfp4(lx2v_ctx *ctx, const uint8_t *packed, const uint8_t *block_scales,
                                       float global_scale, size_t rows, size_t cols, lx2v_weight **out);
LX2V_API void lx2v_weight_free(lx2v_ctx *ctx, lx2v_weight *w);
/* Format, rows, cols and group of a weight. */
LX2V_API lx2v_status lx2v_weight_info(lx2v_ctx *ctx, const lx2v_weight *w, int *format, size_t *rows,
                             size_t *cols, size_t *group);
/* Test hook: the weight dequantized on the device to f32 [rows*cols], with
 * the arithmetic of Q8/Q4/Fp8E4M3::dequantize (quant.rs:180-186, 294-303,
 * 449-455). Bit-exact against those functions. */
LX2V_API lx2v_status lx2v_weight_dequant_f32(lx2v_ctx *ctx, const lx2v_weight *w, float *out);

/* ---- linear (backend.rs:199-212) ----------------------------------------- */
/* Backend::linear:
 *   y[y_row + i, :] = act(x[x_row + i, :] . W^T + bias)   for i < rows
 * x row stride = cols(W) (K), y row stride = rows(W) (N). bias may be NULL
 * (length >= N otherwise). y must not alias x. The product is the exact
 * dequantized weight rounded to bf16 times bf16 activations, accumulated in
 * f32 (the backend's activation rounding, backend.rs:179-181). */
LX2V_API lx2v_status lx2v_linear(lx2v_ctx *ctx, const lx2v_buf *x, size_t x_row, size_t rows,
                        const lx2v_weight *w, const lx2v_buf *bias, int act, lx2v_buf *y,
                        size_t y_row);
/* linear fused with gate_residual (backend.rs:244-253), the sequence of
 * crates/lightx2v-model/src/dit.rs:748-760:
 *   h[h_row + i, j] += act(x[x_row + i, :] . W^T + bias)[j] * mods[gate * N + j]
 * The linear output never goes through an intermediate buffer. */
LX2V_API lx2v_status lx2v_linear_gate_residual(lx2v_ctx *ctx, const lx2v_buf *x, size_t x_row,
                                      size_t rows, const lx2v_weight *w, const lx2v_buf *bias,
                                      int act, lx2v_buf *h, size_t h_row, const lx2v_buf *mods,
                                      size_t gate);
/* Backend::gate_residual (backend.rs:244-253): h[r, j] += a[r, j] * mods[gate*dim + j]. */
LX2V_API lx2v_status lx2v_gate_residual(lx2v_ctx *ctx, lx2v_buf *h, const lx2v_buf *a, size_t rows,
                               size_t dim, const lx2v_buf *mods, size_t gate);

/* ---- attention (backend.rs:275-307) ------------------------------------- */
/* Backend::attention: softmax attention, scale 1/sqrt(head_dim), no mask.
 * q is [heads, sq, head_dim], k and v [heads, sk, head_dim]; out is written
 * with the heads merged, [sq, heads * head_dim] (CPU reference
 * crates/lightx2v-cpu/src/lib.rs:171-208). head_dim 128 with bf16 q/k/v runs
 * on the tensor cores; other head_dims (<= 256) and f32 buffers run a
 * CUDA-core kernel (at most 51,168 keys). */
LX2V_API lx2v_status lx2v_attention(lx2v_ctx *ctx, const lx2v_buf *q, const lx2v_buf *k, const lx2v_buf *v,
                                    size_t heads, size_t sq, size_t sk, size_t head_dim, lx2v_buf *out);
/* Backend::causal_attention: the same with a block mask. `mask` is host
 * memory, [sq][sk] row-major, one byte per pair (nonzero = allowed, the
 * reference's `true`), or NULL (no mask). A query that may see no key gets
 * NaN, as the reference's softmax of an all -inf row does. */
LX2V_API lx2v_status lx2v_causal_attention(lx2v_ctx *ctx, const lx2v_buf *q, const lx2v_buf *k,
                                           const lx2v_buf *v, size_t heads, size_t sq, size_t sk,
                                           size_t head_dim, const uint8_t *mask, lx2v_buf *out);
/* No counterpart in the reference: causal_attention with the mask that
 * LightDit::forward_chunk builds (crates/lightx2v-model/src/dit.rs:645-657),
 * key k visible to query q when tk[k] <= tq[q], given as the temporal
 * indices (host int32 [sq] and [sk]) instead of an sq x sk boolean array.
 * Key blocks that no query of a tile can see are skipped. */
LX2V_API lx2v_status lx2v_causal_attention_temporal(lx2v_ctx *ctx, const lx2v_buf *q, const lx2v_buf *k,
                                                    const lx2v_buf *v, size_t heads, size_t sq, size_t sk,
                                                    size_t head_dim, const int32_t *tq, const int32_t *tk,
                                                    lx2v_buf *out);

/* ---- sparse attention (backend.rs:309-331) ------------------------------- */
/* Backend::sparse_prepare / sparse_attention: LightX2V video sparse attention
 * over a (T, H, W) token grid tiled into 4x4x4 cubes (crates/lightx2v-core/
 * src/sparse.rs), computed as the CPU reference does (cpu lib.rs:496-606):
 * coarse attention over mean-pooled tiles, the top-k key tiles per query tile
 * by the coarse scores (ties to the lower tile), fine attention to the
 * selected tiles' tokens, out = coarse * gate + fine. lx2v_sparse_prepare
 * takes the reference's TilePlan as is: slot_src [num_tiles * 64] (source
 * token per slot, 0xFFFFFFFF padding), block_sizes [num_tiles], the token
 * count, the heads and head_dim of the calls, SparseSpec's topk and scale.
 * q, k, v, gate are [heads, seq, head_dim], out [seq, heads * head_dim]. The
 * fine stage runs the attention kernels with a per-head token mask, so
 * heads * seq^2 bits must stay within 512 MiB (LX2V_ERR_UNSUPPORTED beyond). */
typedef struct lx2v_sparse lx2v_sparse;
LX2V_API lx2v_status lx2v_sparse_prepare(lx2v_ctx *ctx, const uint32_t *slot_src, const uint32_t *block_sizes,
                                         size_t num_tiles, size_t seq, size_t heads, size_t head_dim, size_t topk,
                                         float scale, lx2v_sparse **out);
LX2V_API void lx2v_sparse_free(lx2v_ctx *ctx, lx2v_sparse *sp);
LX2V_API lx2v_status lx2v_sparse_attention(lx2v_ctx *ctx, const lx2v_buf *q, const lx2v_buf *k, const lx2v_buf *v,
                                           const lx2v_buf *gate, const lx2v_sparse *sp, lx2v_buf *out);

/* ---- norms, head_split, patchify, dmd_step (backend.rs:214-273, 392-428) -- */
/* NormKind (backend.rs:47-53): kind 0 = Affine { w, b } (out = LN(x) * w + b,
 * w and b of dim elements), 1 = Mod { scale, shift } (out = LN(x) *
 * (1 + mods[scale]) + mods[shift], rows of the [slots, dim] mods table). */
enum { LX2V_NORM_AFFINE = 0, LX2V_NORM_MOD = 1 };
/* Backend::layer_norm: rows of width dim (at most 4096). Unused arguments of
 * the other kind may be NULL / 0. */
LX2V_API lx2v_status lx2v_layer_norm(lx2v_ctx *ctx, const lx2v_buf *x, size_t rows, size_t dim, int kind,
                                     const lx2v_buf *w, const lx2v_buf *b, size_t scale, size_t shift,
                                     const lx2v_buf *mods, float eps, lx2v_buf *out);
/* Backend::residual_norm: in place h += a * mods[gate] (gate < 0: h += a),
 * then normed = norm(h) of the unrounded f32 sum. */
LX2V_API lx2v_status lx2v_residual_norm(lx2v_ctx *ctx, lx2v_buf *h, const lx2v_buf *a, size_t rows, size_t dim,
                                        const lx2v_buf *mods, long gate, int kind, const lx2v_buf *w,
                                        const lx2v_buf *b, size_t scale, size_t shift, float eps,
                                        lx2v_buf *normed);
/* Backend::head_split: columns [col_off, col_off + heads * head_dim) of src
 * (rows of src_stride) -> out [heads, rows, head_dim], RMS-normalised across
 * all heads times rms_w when rms_w is given, rotated by RoPE on interleaved
 * pairs when cos and sin ([rows, head_dim / 2]) are given. */
LX2V_API lx2v_status lx2v_head_split(lx2v_ctx *ctx, const lx2v_buf *src, size_t rows, size_t src_stride,
                                     size_t col_off, size_t heads, size_t head_dim, const lx2v_buf *rms_w,
                                     const lx2v_buf *cos, const lx2v_buf *sin, float eps, lx2v_buf *out);
/* No counterpart in the reference (its head_split normalises across the
 * heads it is given, all of them): for a tensor-parallel block that holds
 * only some heads. lx2v_row_sumsq writes out[r] = sum of the squares of
 * columns [col_off, col_off + width) of row r (f32 [rows]); the caller sums
 * these over the ranks (lx2v_all_reduce_sum) and lx2v_head_split_rms then
 * normalises by rsqrt(sumsq[r] / rms_dim + eps), rms_dim being the width of
 * all heads together, so that every rank's heads are normalised exactly as
 * head_split normalises the full row. */
LX2V_API lx2v_status lx2v_row_sumsq(lx2v_ctx *ctx, const lx2v_buf *src, size_t rows, size_t src_stride,
                                    size_t col_off, size_t width, lx2v_buf *out);
LX2V_API lx2v_status lx2v_head_split_rms(lx2v_ctx *ctx, const lx2v_buf *src, size_t rows, size_t src_stride,
                                         size_t col_off, size_t heads, size_t head_dim, const lx2v_buf *rms_w,
                                         const lx2v_buf *sumsq, size_t rms_dim, const lx2v_buf *cos,
                                         const lx2v_buf *sin, float eps, lx2v_buf *out);
/* Backend::patchify: latent [c, t, h, w] -> tokens [t*(h/p)*(w/p), c*p*p],
 * feature c*p^2 + kh*p + kw. */
/* lx2v_head_split_rms with the row statistic summed from `parts` slices of
 * sumsq ([parts][rows], added in order): the slices are the ranks' sums from
 * lx2v_row_sumsq_peers. */
LX2V_API lx2v_status lx2v_head_split_rms_parts(lx2v_ctx *ctx, const lx2v_buf *src, size_t rows, size_t src_stride,
                                               size_t col_off, size_t heads, size_t head_dim, const lx2v_buf *rms_w,
                                               const lx2v_buf *sumsq, size_t parts, size_t rms_dim,
                                               const lx2v_buf *cos, const lx2v_buf *sin, float eps, lx2v_buf *out);
LX2V_API lx2v_status lx2v_patchify(lx2v_ctx *ctx, const lx2v_buf *latent, size_t c, size_t t, size_t h, size_t w,
                                   size_t p, lx2v_buf *out);
/* Backend::unpatchify: the inverse of lx2v_patchify. */
LX2V_API lx2v_status lx2v_unpatchify(lx2v_ctx *ctx, const lx2v_buf *x, size_t c, size_t t, size_t h, size_t w,
                                     size_t p, lx2v_buf *out);
/* Backend::dmd_step: in place on x[0..n): x0 = x - sigma_t * v, then
 * x = (1 - sigma_next) * x0 + sigma_next * noise when noise is given. */
LX2V_API lx2v_status lx2v_dmd_step(lx2v_ctx *ctx, lx2v_buf *x, const lx2v_buf *v, const lx2v_buf *noise,
                                   float sigma_t, float sigma_next, size_t n);

/* ---- KV cache / MemRoPE (backend.rs:334-390) ---------------------------- */
/* The per-layer KV cache (Backend::KvCache; CPU reference
 * crates/lightx2v-cpu/src/lib.rs:607-806). K and V rows live on the device
 * as [heads][capacity][head_dim] bf16; each row carries a temporal index and
 * a slot kind (sink, long EMA, short EMA, recent, new) kept on the host. */
typedef struct lx2v_kv_cache lx2v_kv_cache;
/* Backend::kv_cache_new: an empty cache with room for capacity_tokens rows
 * (it grows when a MemRoPE update needs more). */
LX2V_API lx2v_status lx2v_kv_cache_new(lx2v_ctx *ctx, size_t heads, size_t head_dim, size_t capacity_tokens,
                                       lx2v_kv_cache **out);
LX2V_API void lx2v_kv_cache_free(lx2v_ctx *ctx, lx2v_kv_cache *cache);
/* Backend::kv_cache_append: k and v are [heads, rows, head_dim] buffers,
 * temporal host [rows]; the rows are appended as New slots. */
LX2V_API lx2v_status lx2v_kv_cache_append(lx2v_ctx *ctx, lx2v_kv_cache *cache, const lx2v_buf *k,
                                          const lx2v_buf *v, size_t rows, const size_t *temporal);
/* Backend::kv_cache_put: overwrite the rows already cached under the same
 * temporal indices (the same chunk on the next denoising step), else
 * append. */
LX2V_API lx2v_status lx2v_kv_cache_put(lx2v_ctx *ctx, lx2v_kv_cache *cache, const lx2v_buf *k, const lx2v_buf *v,
                                       size_t rows, const size_t *temporal);
/* Backend::kv_cache_len. */
LX2V_API lx2v_status lx2v_kv_cache_len(lx2v_ctx *ctx, const lx2v_kv_cache *cache, size_t *rows);
/* Backend::kv_cache_temporal: the rows' temporal indices in cache order into
 * out[0..rows) (cap >= rows). */
LX2V_API lx2v_status lx2v_kv_cache_temporal(lx2v_ctx *ctx, const lx2v_kv_cache *cache, size_t *out, size_t cap);
/* Backend::kv_cache_kv: the cached K and V as [heads, rows, head_dim] into
 * k_out / v_out (bf16 or f32 buffers of at least heads * rows * head_dim). */
LX2V_API lx2v_status lx2v_kv_cache_kv(lx2v_ctx *ctx, const lx2v_kv_cache *cache, lx2v_buf *k_out,
                                      lx2v_buf *v_out);
/* Backend::kv_cache_memrope_update with the MemRopeConfig fields it reads
 * (crates/lightx2v-core/src/config.rs:265-300; new_frames is
 * MemRopeConfig::new_frames()): seed the EMA slots, graduate New frames to
 * Recent, and while more than cache_frames frames are cached fold the
 * oldest Recent (else New) frame into the EMA slots and evict it. */
LX2V_API lx2v_status lx2v_kv_cache_memrope_update(lx2v_ctx *ctx, lx2v_kv_cache *cache, size_t cache_frames,
                                                  size_t sink_frames, size_t new_frames, float ema_alpha_long,
                                                  float ema_alpha_short, size_t frame_tokens);
/* No counterpart in the reference (there: kv_cache_kv, then causal_attention
 * with the boolean mask, crates/lightx2v-model/src/dit.rs:643-667): the
 * causal attention of q ([heads, sq, head_dim]) against the cache, reading
 * K and V in place, key visible to query i when its temporal index <= tq[i]
 * (host int32 [sq]). out is [sq, heads * head_dim]. */
LX2V_API lx2v_status lx2v_kv_cache_attention(lx2v_ctx *ctx, const lx2v_buf *q, size_t sq, const int32_t *tq,
                                             const lx2v_kv_cache *cache, lx2v_buf *out);

/* ---- profiling (backend.rs:192-196) -------------------------------------- */
/* Backend::profile_report: per-op device time since the last reset, as JSON
 * {"op": {"calls": n, "ms": t}, ...}. Profiling is on when the context was
 * created with LIGHTX2V_PROFILE set to anything but "0" (the reference's
 * switch, crates/lightx2v-cpu/src/lib.rs:27-34). `written` gets the length
 * needed including the NUL. */
LX2V_API lx2v_status lx2v_profile_json(lx2v_ctx *ctx, char *buf, size_t cap, size_t *written);
/* Backend::profile_reset. */
LX2V_API lx2v_status lx2v_profile_reset(lx2v_ctx *ctx);

/* Size of the scratch array behind lx2v_linear_noalloc: 10 MiB, held on
 * every GPU that loads this library, for the whole life of the process. */
#define LX2V_NOALLOC_SCRATCH_BYTES (10u * 1024u * 1024u)

/* lx2v_linear without any device allocation. No counterpart in the
 * reference (lightx2v-rs has no GPU linear; this is an addition for callers
 * of this library). For callers that cannot let the library call cudaMalloc
 * while they run: a serving loop whose device memory was planned up front
 * and must not grow mid-request, or a caller for whom cudaMalloc's implicit
 * device-wide synchronisation would stall other streams.
 * Same arguments and result as lx2v_linear (no gated residual); it always
 * runs the CTA-pair tensor-core kernel with a stream-K split, and keeps the
 * split's partial tiles in a fixed array of LX2V_NOALLOC_SCRATCH_BYTES inside
 * the library instead of a context workspace.
 * - The first call on a device looks up that array's device address
 *   (cudaGetSymbolAddress); make that first call before any stream capture.
 * - Every call on a device shares the array: calls whose kernels may overlap
 *   on the GPU (other streams or contexts on the same device) race and give
 *   wrong results. Serialise them.
 * - LX2V_ERR_UNSUPPORTED when the shape cannot use the tensor-core kernel
 *   (x not bf16, K or N not a multiple of 16, fewer than 16 rows, ...) or the
 *   GPU has so many SMs that its partial tiles would not fit the array. */
LX2V_API lx2v_status lx2v_linear_noalloc(lx2v_ctx *ctx, const lx2v_buf *x, size_t x_row, size_t rows,
                                         const lx2v_weight *w, const lx2v_buf *bias, int act, lx2v_buf *y,
                                         size_t y_row);

/* ---- tensor parallelism ---------------------------------------------------- */
/* No counterpart in the reference (its backends run on one device). One
 * process per GPU: rank 0 makes an id, every rank of the group passes the
 * same bytes to lx2v_comm_init (exchanged by the caller, e.g. through its
 * launcher's store), and lx2v_all_reduce_sum then sums a buffer over the
 * group on the context's stream (NCCL over NVLink; f32 or bf16). NCCL is
 * opened on first use (libnccl.so.2); without it these calls return
 * LX2V_ERR_UNSUPPORTED. */
#define LX2V_COMM_ID_BYTES 128
LX2V_API lx2v_status lx2v_comm_unique_id(unsigned char *out, size_t cap);
LX2V_API lx2v_status lx2v_comm_init(lx2v_ctx *ctx, const unsigned char *id, int rank, int world);
/* buf[0..len) = sum over the group's ranks of their buf[0..len), in place. */
LX2V_API lx2v_status lx2v_all_reduce_sum(lx2v_ctx *ctx, lx2v_buf *buf, size_t len);

/* ---- tensor parallelism over NVLink peer memory ---------------------------- */
/* No counterpart in the reference (it runs on one device). A row-split
 * linear of a DiT block leaves every rank with a partial product of all M
 * rows; with the ranks' buffers shared by CUDA IPC, lx2v_tp_reduce_norm does
 * the reduce-scatter, the residual add, the norm and the all-gather in one
 * kernel per rank, and lx2v_peers_barrier orders the ranks around it.
 *
 * lx2v_buf_ipc_handle writes the CUDA IPC handle of an own buffer (at most
 * LX2V_IPC_HANDLE_BYTES bytes); the caller sends it to the other processes of
 * the group (as it does the NCCL id), and lx2v_buf_open_ipc maps a peer's
 * buffer into this context (len elements of dtype; lx2v_buf_free unmaps it).
 * Peer buffers are device memory of another GPU: only the calls below and
 * lx2v_tp_reduce_norm's arguments may take them. */
#define LX2V_IPC_HANDLE_BYTES 64
LX2V_API lx2v_status lx2v_buf_ipc_handle(lx2v_ctx *ctx, const lx2v_buf *buf, unsigned char *out, size_t cap);
LX2V_API lx2v_status lx2v_buf_open_ipc(lx2v_ctx *ctx, const unsigned char *handle, size_t len, int dtype,
                                       lx2v_buf **out);
/* A group of `world` ranks (at most 8, one process per GPU), this one being
 * `rank`. flag_bufs[r] is rank r's flag buffer as this context sees it (its
 * own buffer at index rank, peers' opened by lx2v_buf_open_ipc): every rank
 * allocates one of at least world u32 (e.g. world f32 elements, zeroed by
 * lx2v_buf_alloc) before any rank's first barrier. */
typedef struct lx2v_peers lx2v_peers;
LX2V_API lx2v_status lx2v_peers_create(lx2v_ctx *ctx, int rank, int world, lx2v_buf *const *flag_bufs,
                                       lx2v_peers **out);
LX2V_API void lx2v_peers_free(lx2v_peers *g);
/* Barrier on the context's stream: work queued after it on any rank sees the
 * writes (local and to peer memory) of work queued before it on every rank.
 * Every rank calls the group's barriers in the same order. The wait is
 * bounded (lx2v_set_wait_limit_ns); on expiry the next lx2v_sync returns
 * LX2V_ERR_DEVICE. */
LX2V_API lx2v_status lx2v_peers_barrier(lx2v_ctx *ctx, lx2v_peers *g);
/* Rows [row0, row1) of an M x dim block output owned by this rank:
 *   h[r] += mods[gate] * sum over ranks p (in rank order, f32) of parts[p][r]
 *   (gate < 0: h[r] += the sum; parts NULL: no add), then
 *   normed[p][r] = norm(h[r]) for every rank p,
 * norm as lx2v_layer_norm (kind 0 affine w, b; 1 modulated by norm_mods rows
 * scale, shift). h is f32; parts and normed are indexed by rank (own buffer
 * at index rank, peers' opened by IPC). The caller puts a barrier before (the
 * partials are complete) and after (the outputs are). Replaces the
 * reference's residual_norm (cpu lib.rs:364-392), or gate_residual followed by
 * layer_norm, on a block split over the group's GPUs. */
/* lx2v_row_sumsq over the group: this rank's row sums of squares of columns
 * [col_off, col_off + width) into outs[p][rank * rows + r] for every rank p
 * (each out f32 of world * rows; own buffer at index rank, peers' by IPC).
 * After a barrier, lx2v_head_split_rms_parts with parts = world adds the
 * ranks' sums in rank order: the cross-head q/k RMS of a head-split block
 * without a collective library. */
LX2V_API lx2v_status lx2v_row_sumsq_peers(lx2v_ctx *ctx, lx2v_peers *g, const lx2v_buf *src, size_t rows,
                                          size_t src_stride, size_t col_off, size_t width, lx2v_buf *const *outs);
LX2V_API lx2v_status lx2v_tp_reduce_norm(lx2v_ctx *ctx, lx2v_peers *g, lx2v_buf *const *parts, lx2v_buf *h,
                                         size_t row0, size_t row1, size_t dim, const lx2v_buf *gate_mods, long gate,
                                         int kind, const lx2v_buf *w, const lx2v_buf *b, const lx2v_buf *norm_mods,
                                         size_t scale, size_t shift, float eps, lx2v_buf *const *normed);

/* ---- knobs for tests and benchmarks -------------------------------------- */
/* Kernel choice for linear: 0 = automatic, 1 = tensor-core GEMM (tcgen05, one
 * CTA per tile), 2 = small-M GEMV, 3 = generic CUDA-core kernel, 4 = tensor-
 * core GEMM on CTA pairs (tcgen05 cta_group::2), 5 = two-pass (weight decoded
 * to bf16, then a CTA-pair GEMM with both operands in shared memory). A
 * forced choice that cannot run the shape returns LX2V_ERR_UNSUPPORTED. */
LX2V_API lx2v_status lx2v_set_linear_path(lx2v_ctx *ctx, int path);
/* Token tile of the tensor-core kernel: 0 = automatic, else 128, 192 or 256
 * tokens per tile (each tile is 128 output features wide). */
LX2V_API lx2v_status lx2v_set_token_tile(lx2v_ctx *ctx, int tokens);
/* Work split of the CTA-pair kernel: 0 = automatic (whole tiles; for the
 * two-pass kernel's gated residual into an f32 buffer, tiles may be cut into
 * k-ranges that each reduce-add into it), 1 = whole tiles per pair, 2 =
 * stream-K (equal k-block ranges per pair; a tile split between pairs is
 * summed through a context-owned workspace, allocated on first use).
 * No reference counterpart: lightx2v-rs has no GPU GEMM to tune. */
LX2V_API lx2v_status lx2v_set_split_mode(lx2v_ctx *ctx, int mode);
/* Bounded-wait limit of the pipelined kernels, in nanoseconds (default 2e9).
 * A wait that expires makes the kernel stop and record an error that the
 * next lx2v_sync returns as LX2V_ERR_DEVICE. */
LX2V_API lx2v_status lx2v_set_wait_limit_ns(lx2v_ctx *ctx, uint64_t ns);
/* Kernels this context has launched (for launch accounting in benchmarks). */
LX2V_API lx2v_status lx2v_launch_count(lx2v_ctx *ctx, uint64_t *count);

#ifdef __cplusplus
}
#endif
#endif /* LIGHTX2V_CUDA_H */
