// dit_ops.cu — the DiT block's row-wise and elementwise ops around the
// linears and the attention: layer_norm / residual_norm (AdaLN or affine),
// head_split (RMS across all heads, per-channel weight, interleaved RoPE,
// [rows, heads*d] -> [heads, rows, d]), patchify / unpatchify and dmd_step.
// CPU reference: crates/lightx2v-cpu/src/lib.rs:328-459 and 806-874; trait
// crates/lightx2v-core/src/backend.rs:214-273, 392-428.
//
// All of them are HBM-bound: the row is held in registers between its two
// passes (statistics, then the normalised output), so each row is read once
// and written once. Rows of 256 G values (G up to 12) run one warp per row;
// other widths one CTA per row.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include "dit_ops.h"

namespace lx2v {

namespace {

constexpr int ROW_THREADS = 128;
constexpr int ROW_PER_THREAD = 32;  // rows up to 4096 values

__device__ __forceinline__ float ld_v(const void *p, int f32, int64_t i) {
    return f32 ? reinterpret_cast<const float *>(p)[i] : __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[i]);
}
__device__ __forceinline__ void st_v(void *p, int f32, int64_t i, float v) {
    if (f32) reinterpret_cast<float *>(p)[i] = v;
    else reinterpret_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v);
}

// Sum over the CTA (ROW_THREADS threads); every thread gets the total.
__device__ __forceinline__ float block_sum(float v, float *red) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    __syncthreads();  // red is free (an earlier call has read it)
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < ROW_THREADS / 32; ++w) t += red[w];
    return t;
}

// One row: mean and variance of vals[0..n) (thread's share), then the
// normalised values written to out (row r). Norm kind 0 = affine (w, b),
// 1 = modulated (1 + mods[scale]) and + mods[shift].
__device__ __forceinline__ void norm_row(const float (&vals)[ROW_PER_THREAD], const NormArgs &a, int64_t r,
                                         float *red) {
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < ROW_PER_THREAD; ++i)
        if (threadIdx.x + i * ROW_THREADS < a.dim) s += vals[i];
    const float mean = block_sum(s, red) / (float)a.dim;
    float vs = 0.0f;
#pragma unroll
    for (int i = 0; i < ROW_PER_THREAD; ++i)
        if (threadIdx.x + i * ROW_THREADS < a.dim) {
            const float c = vals[i] - mean;
            vs += c * c;
        }
    const float var = block_sum(vs, red) / (float)a.dim;
    const float inv = 1.0f / sqrtf(var + a.eps);
#pragma unroll
    for (int i = 0; i < ROW_PER_THREAD; ++i) {
        const int j = threadIdx.x + i * ROW_THREADS;
        if (j >= a.dim) break;
        const float n = (vals[i] - mean) * inv;
        float o;
        if (a.kind == 0) o = n * ld_v(a.w, a.w_f32, j) + ld_v(a.b, a.b_f32, j);
        else o = n * (1.0f + ld_v(a.mods, a.mods_f32, (int64_t)a.scale * a.dim + j)) +
                 ld_v(a.mods, a.mods_f32, (int64_t)a.shift * a.dim + j);
        st_v(a.out, a.out_f32, r * a.dim + j, o);
    }
}

__global__ void __launch_bounds__(ROW_THREADS) layer_norm_kernel(NormArgs a) {
    __shared__ float red[ROW_THREADS / 32];
    const int64_t r = blockIdx.x;
    float vals[ROW_PER_THREAD];
#pragma unroll
    for (int i = 0; i < ROW_PER_THREAD; ++i) {
        const int j = threadIdx.x + i * ROW_THREADS;
        vals[i] = j < a.dim ? ld_v(a.x, a.x_f32, r * a.dim + j) : 0.0f;
    }
    norm_row(vals, a, r, red);
}

// h += a * mods[gate] (or + a), stored back, then the norm of the f32 sum.
__global__ void __launch_bounds__(ROW_THREADS) residual_norm_kernel(NormArgs a, void *h, int h_f32, const void *res,
                                                                    int res_f32, int gate) {
    __shared__ float red[ROW_THREADS / 32];
    const int64_t r = blockIdx.x;
    float vals[ROW_PER_THREAD];
#pragma unroll
    for (int k = 0; k < ROW_PER_THREAD; ++k) {
        const int j = threadIdx.x + k * ROW_THREADS;
        vals[k] = 0.0f;
        if (j < a.dim) {
            const int64_t i = r * a.dim + j;
            const float g = gate >= 0 ? ld_v(a.mods, a.mods_f32, (int64_t)gate * a.dim + j) : 1.0f;
            const float v = ld_v(h, h_f32, i) + ld_v(res, res_f32, i) * g;
            st_v(h, h_f32, i, v);
            vals[k] = v;
        }
    }
    norm_row(vals, a, r, red);
}

// Row r's sum of squares over all heads: the parts (one per rank) added in order.
__device__ __forceinline__ float summed_sumsq(const HeadSplitArgs &a, int64_t r) {
    float t = 0.0f;
    for (int p = 0; p < a.sumsq_parts; ++p) t += a.sumsq[p * a.sumsq_stride + r];
    return t;
}

// One row of src: columns [col_off, col_off + heads * hd), optional RMS over
// all of them times w[j], optional RoPE on interleaved pairs of each head,
// written to out[h][r][:]. Thread t takes the pairs t, t + 128, ...
__global__ void __launch_bounds__(ROW_THREADS) head_split_kernel(HeadSplitArgs a) {
    __shared__ float red[ROW_THREADS / 32];
    const int64_t r = blockIdx.x;
    const int d = a.heads * a.head_dim;
    const int pairs = d / 2;
    constexpr int NP = ROW_PER_THREAD / 2;
    float x0[NP], x1[NP];
    const int64_t base = r * a.src_stride + a.col_off;
#pragma unroll
    for (int i = 0; i < NP; ++i) {
        const int pi = threadIdx.x + i * ROW_THREADS;
        x0[i] = pi < pairs ? ld_v(a.src, a.src_f32, base + 2 * pi) : 0.0f;
        x1[i] = pi < pairs ? ld_v(a.src, a.src_f32, base + 2 * pi + 1) : 0.0f;
    }
    if (a.rms_w) {
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < NP; ++i) ss += x0[i] * x0[i] + x1[i] * x1[i];  // zeros past the row add nothing
        const float ms = a.sumsq ? summed_sumsq(a, r) / (float)a.rms_dim : block_sum(ss, red) / (float)d;
        const float inv = 1.0f / sqrtf(ms + a.eps);
#pragma unroll
        for (int i = 0; i < NP; ++i) {
            const int j = 2 * (threadIdx.x + i * ROW_THREADS);
            if (j >= d) break;
            x0[i] = x0[i] * inv * ld_v(a.rms_w, a.w_f32, j);
            x1[i] = x1[i] * inv * ld_v(a.rms_w, a.w_f32, j + 1);
        }
    }
#pragma unroll
    for (int i = 0; i < NP; ++i) {
        const int j = 2 * (threadIdx.x + i * ROW_THREADS);
        if (j >= d) break;
        const int h = j / a.head_dim, e = j % a.head_dim;
        float o0 = x0[i], o1 = x1[i];
        if (a.cos) {
            const int64_t ci = r * (a.head_dim / 2) + e / 2;
            const float c = ld_v(a.cos, a.cs_f32, ci), sn = ld_v(a.sin, a.cs_f32, ci);
            o0 = x0[i] * c - x1[i] * sn;
            o1 = x0[i] * sn + x1[i] * c;
        }
        const int64_t oi = ((int64_t)h * a.rows + r) * a.head_dim + e;
        st_v(a.out, a.out_f32, oi, o0);
        st_v(a.out, a.out_f32, oi + 1, o1);
    }
}

// latent [c, t, h, w] <-> tokens [t * (h/p) * (w/p), c * p * p]; `to_tokens`
// picks the direction. Thread = one element of the token matrix.
__global__ void patchify_kernel(const void *src, int src_f32, void *dst, int dst_f32, int c, int t, int h, int w, int p,
                                int to_tokens) {
    const int hp = h / p, wp = w / p, feat = c * p * p;
    const int64_t total = (int64_t)t * hp * wp * feat;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t tok = i / feat;
        const int f = (int)(i % feat);
        const int cc = f / (p * p), kh = (f / p) % p, kw = f % p;
        const int ww = (int)(tok % wp), hh = (int)((tok / wp) % hp), tt = (int)(tok / ((int64_t)wp * hp));
        const int64_t li = (((int64_t)cc * t + tt) * h + hh * p + kh) * w + ww * p + kw;
        if (to_tokens) st_v(dst, dst_f32, i, ld_v(src, src_f32, li));
        else st_v(dst, dst_f32, li, ld_v(src, src_f32, i));
    }
}

// x = x - sigma_t * v, then (1 - sigma_next) * x0 + sigma_next * noise.
__global__ void dmd_step_kernel(void *x, int x_f32, const void *v, int v_f32, const void *noise, int n_f32,
                                float sigma_t, float sigma_next, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float x0 = ld_v(x, x_f32, i) - sigma_t * ld_v(v, v_f32, i);
        st_v(x, x_f32, i, noise ? (1.0f - sigma_next) * x0 + sigma_next * ld_v(noise, n_f32, i) : x0);
    }
}

// ---- vectorized row kernels: thread t owns values [8t, 8t + 8) of the row ----
// (dim a multiple of 256, at most 4096: blockDim = dim / 8 is whole warps)
__device__ __forceinline__ void ld8(const void *p, int f32, int64_t i, float (&v)[8]) {
    if (f32) {
        const float4 a = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(p) + i);
        const float4 b = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(p) + i + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
        const uint4 u = *reinterpret_cast<const uint4 *>(reinterpret_cast<const __nv_bfloat16 *>(p) + i);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            v[2 * k] = __uint_as_float(w[k] << 16);
            v[2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
        }
    }
}
__device__ __forceinline__ void st8(void *p, int f32, int64_t i, const float (&v)[8]) {
    if (f32) {
        float4 *d = reinterpret_cast<float4 *>(reinterpret_cast<float *>(p) + i);
        d[0] = make_float4(v[0], v[1], v[2], v[3]);
        d[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
        uint32_t w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const __nv_bfloat162 b = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
            w[k] = *reinterpret_cast<const uint32_t *>(&b);
        }
        *reinterpret_cast<uint4 *>(reinterpret_cast<__nv_bfloat16 *>(p) + i) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

__device__ __forceinline__ float block_sum_any(float v, float *red) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.0f;
    const int nw = (int)(blockDim.x >> 5);
    for (int w = 0; w < nw; ++w) t += red[w];
    return t;
}

template <bool RESID>
__global__ void __launch_bounds__(512) norm_vec_kernel(NormArgs a, void *h, int h_f32, const void *res, int res_f32,
                                                       int gate) {
    __shared__ float red[16];
    const int64_t r = blockIdx.x;
    const int j0 = threadIdx.x * 8;
    const int64_t i0 = r * a.dim + j0;
    float v[8];
    if (RESID) {
        float hv[8], av[8], g[8];
        ld8(h, h_f32, i0, hv);
        ld8(res, res_f32, i0, av);
        if (gate >= 0) ld8(a.mods, a.mods_f32, (int64_t)gate * a.dim + j0, g);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = hv[k] + av[k] * (gate >= 0 ? g[k] : 1.0f);
        st8(h, h_f32, i0, v);
    } else {
        ld8(a.x, a.x_f32, i0, v);
    }
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) s += v[k];
    const float mean = block_sum_any(s, red) / (float)a.dim;
    float vs = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const float c = v[k] - mean;
        vs += c * c;
    }
    const float var = block_sum_any(vs, red) / (float)a.dim;
    const float inv = 1.0f / sqrtf(var + a.eps);
    float p[8], q[8], o[8];
    if (a.kind == 0) {
        ld8(a.w, a.w_f32, j0, p);
        ld8(a.b, a.b_f32, j0, q);
#pragma unroll
        for (int k = 0; k < 8; ++k) o[k] = (v[k] - mean) * inv * p[k] + q[k];
    } else {
        ld8(a.mods, a.mods_f32, (int64_t)a.scale * a.dim + j0, p);
        ld8(a.mods, a.mods_f32, (int64_t)a.shift * a.dim + j0, q);
#pragma unroll
        for (int k = 0; k < 8; ++k) o[k] = (v[k] - mean) * inv * (1.0f + p[k]) + q[k];
    }
    st8(a.out, a.out_f32, i0, o);
}

// head_split with 8 values (4 RoPE pairs of one head) per thread.
__global__ void __launch_bounds__(512) head_split_vec_kernel(HeadSplitArgs a) {
    __shared__ float red[16];
    const int64_t r = blockIdx.x;
    const int d = a.heads * a.head_dim;
    const int j0 = threadIdx.x * 8;
    float x[8];
    ld8(a.src, a.src_f32, r * a.src_stride + a.col_off + j0, x);
    if (a.rms_w) {
        float ss = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; ++k) ss += x[k] * x[k];
        const float ms = a.sumsq ? summed_sumsq(a, r) / (float)a.rms_dim : block_sum_any(ss, red) / (float)d;
        const float inv = 1.0f / sqrtf(ms + a.eps);
        float w[8];
        ld8(a.rms_w, a.w_f32, j0, w);
#pragma unroll
        for (int k = 0; k < 8; ++k) x[k] = x[k] * inv * w[k];
    }
    const int h = j0 / a.head_dim, e = j0 % a.head_dim;
    float o[8];
    if (a.cos) {
        const int64_t ci = r * (a.head_dim / 2) + e / 2;
        float c[4], sn[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            c[k] = ld_v(a.cos, a.cs_f32, ci + k);
            sn[k] = ld_v(a.sin, a.cs_f32, ci + k);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            o[2 * k] = x[2 * k] * c[k] - x[2 * k + 1] * sn[k];
            o[2 * k + 1] = x[2 * k] * sn[k] + x[2 * k + 1] * c[k];
        }
    } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) o[k] = x[k];
    }
    st8(a.out, a.out_f32, ((int64_t)h * a.rows + r) * a.head_dim + e, o);
}

// ---- one warp per row (8 rows a CTA) --------------------------------------
// For rows of 256 G values: lane l holds the groups of 8 values l, l + 32,
// ..., so every lane has G 16-byte loads in flight and the row statistics are
// warp shuffles, not CTA barriers (the one-CTA-per-row kernels above were
// latency-bound at 1.6-3.7 TB/s on the chunk's rows).
constexpr int WROWS = 8;

__device__ __forceinline__ float warp_sum(float v) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}
__device__ __forceinline__ void unpack8(const uint4 u, float (&v)[8]) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        v[2 * k] = __uint_as_float(w[k] << 16);
        v[2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
    }
}

// head_split of a bf16 source row (the same arithmetic as head_split_vec_kernel).
template <int G>
__global__ void __launch_bounds__(32 * WROWS) head_split_warp_kernel(HeadSplitArgs a) {
    const int lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * WROWS + (threadIdx.x >> 5);
    if (r >= a.rows) return;  // whole warps leave together
    const int d = 256 * G;
    const __nv_bfloat16 *src = reinterpret_cast<const __nv_bfloat16 *>(a.src) + r * a.src_stride + a.col_off;
    uint4 raw[G];
#pragma unroll
    for (int g = 0; g < G; ++g) raw[g] = *reinterpret_cast<const uint4 *>(src + (g * 32 + lane) * 8);
    float inv = 1.0f;
    if (a.rms_w) {
        float ss = 0.0f;
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float x[8];
            unpack8(raw[g], x);
#pragma unroll
            for (int k = 0; k < 8; ++k) ss += x[k] * x[k];
        }
        const float ms = a.sumsq ? summed_sumsq(a, r) / (float)a.rms_dim : warp_sum(ss) / (float)d;
        inv = 1.0f / sqrtf(ms + a.eps);
    }
    const int hd = a.head_dim;
    // when head_dim divides 256, a lane's 8 values sit at the same offset of
    // their head in every group: its RoPE angles are loaded once, before any
    // store (a load after a store cannot be moved above it)
    const bool rope_once = a.cos && 256 % hd == 0;
    float c1[4], s1[4];
    if (rope_once) {
        const int64_t ci = r * (hd / 2) + ((lane * 8) % hd) / 2;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            c1[k] = ld_v(a.cos, a.cs_f32, ci + k);
            s1[k] = ld_v(a.sin, a.cs_f32, ci + k);
        }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const int j0 = (g * 32 + lane) * 8;
        float x[8];
        unpack8(raw[g], x);
        if (a.rms_w) {
            float w[8];
            ld8(a.rms_w, a.w_f32, j0, w);
#pragma unroll
            for (int k = 0; k < 8; ++k) x[k] = x[k] * inv * w[k];
        }
        const int h = j0 / hd, e = j0 % hd;
        float o[8];
        if (a.cos) {
            const int64_t ci = r * (hd / 2) + e / 2;
            float c[4], sn[4];
            if (rope_once) {
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    c[k] = c1[k];
                    sn[k] = s1[k];
                }
            } else if (a.cs_f32) {
                const float4 c4 = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(a.cos) + ci);
                const float4 s4 = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(a.sin) + ci);
                c[0] = c4.x; c[1] = c4.y; c[2] = c4.z; c[3] = c4.w;
                sn[0] = s4.x; sn[1] = s4.y; sn[2] = s4.z; sn[3] = s4.w;
            } else {
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    c[k] = ld_v(a.cos, 0, ci + k);
                    sn[k] = ld_v(a.sin, 0, ci + k);
                }
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                o[2 * k] = x[2 * k] * c[k] - x[2 * k + 1] * sn[k];
                o[2 * k + 1] = x[2 * k] * sn[k] + x[2 * k + 1] * c[k];
            }
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) o[k] = x[k];
        }
        st8(a.out, a.out_f32, ((int64_t)h * a.rows + r) * hd + e, o);
    }
}

// layer_norm (RESID false) / residual_norm (RESID true) of a row of 256 G
// values (the same arithmetic as norm_vec_kernel).
template <int G, bool RESID>
__global__ void __launch_bounds__(32 * WROWS) norm_warp_kernel(NormArgs a, void *h, int h_f32, const void *res,
                                                              int res_f32, int gate) {
    const int lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * WROWS + (threadIdx.x >> 5);
    if (r >= a.rows) return;
    float v[G][8];
    // every load of the row first, then the stores to h (a load after a store
    // to a buffer that may alias it could not be moved above the store)
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const int j0 = (g * 32 + lane) * 8;
        const int64_t i0 = r * a.dim + j0;
        if (RESID) {
            float av[8], gg[8];
            ld8(h, h_f32, i0, v[g]);
            ld8(res, res_f32, i0, av);
            if (gate >= 0) ld8(a.mods, a.mods_f32, (int64_t)gate * a.dim + j0, gg);
#pragma unroll
            for (int k = 0; k < 8; ++k) v[g][k] = v[g][k] + av[k] * (gate >= 0 ? gg[k] : 1.0f);
        } else {
            ld8(a.x, a.x_f32, i0, v[g]);
        }
    }
    if (RESID) {
#pragma unroll
        for (int g = 0; g < G; ++g) st8(h, h_f32, r * a.dim + (g * 32 + lane) * 8, v[g]);
    }
    float s = 0.0f;
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int k = 0; k < 8; ++k) s += v[g][k];
    const float mean = warp_sum(s) / (float)a.dim;
    float vs = 0.0f;
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float c = v[g][k] - mean;
            vs += c * c;
        }
    const float var = warp_sum(vs) / (float)a.dim;
    const float inv = 1.0f / sqrtf(var + a.eps);
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const int j0 = (g * 32 + lane) * 8;
        float p[8], q[8], o[8];
        if (a.kind == 0) {
            ld8(a.w, a.w_f32, j0, p);
            ld8(a.b, a.b_f32, j0, q);
#pragma unroll
            for (int k = 0; k < 8; ++k) o[k] = (v[g][k] - mean) * inv * p[k] + q[k];
        } else {
            ld8(a.mods, a.mods_f32, (int64_t)a.scale * a.dim + j0, p);
            ld8(a.mods, a.mods_f32, (int64_t)a.shift * a.dim + j0, q);
#pragma unroll
            for (int k = 0; k < 8; ++k) o[k] = (v[g][k] - mean) * inv * (1.0f + p[k]) + q[k];
        }
        st8(a.out, a.out_f32, r * a.dim + j0, o);
    }
}

// One row per CTA: the sum of squares of `width` values, f32.
__global__ void __launch_bounds__(ROW_THREADS) row_sumsq_kernel(const void *src, int src_f32, int64_t stride,
                                                                int64_t col_off, int width, float *out) {
    __shared__ float red[ROW_THREADS / 32];
    const int64_t r = blockIdx.x;
    float ss = 0.0f;
    for (int j = threadIdx.x; j < width; j += ROW_THREADS) {
        const float v = ld_v(src, src_f32, r * stride + col_off + j);
        ss += v * v;
    }
    const float t = block_sum(ss, red);
    if (threadIdx.x == 0) out[r] = t;
}

int grid_elems(int64_t n) {
    int64_t b = (n + 255) / 256;
    return (int)(b < 1 ? 1 : (b > 148 * 32 ? 148 * 32 : b));
}

}  // namespace

bool row_op_supported(int dim) { return dim > 0 && dim <= ROW_THREADS * ROW_PER_THREAD; }

// The vectorized kernels need whole warps of 8-value threads and 16-byte
// aligned rows (every buffer and row offset here is a multiple of 16 bytes
// when dim % 256 == 0).
static bool vec_ok(int dim) { return dim % 256 == 0 && dim <= 4096; }

// Warp-per-row instantiations: rows of 256 G values.
template <bool RESID>
static bool norm_warp_launch(const NormArgs &a, void *h, int h_f32, const void *res, int res_f32, int gate,
                             cudaStream_t st) {
    if (a.dim % 256 != 0) return false;
    const unsigned grid = (unsigned)((a.rows + WROWS - 1) / WROWS);
    switch (a.dim / 256) {
#define LX2V_NORM_G(G)                                                                                  \
    case G:                                                                                             \
        norm_warp_kernel<G, RESID><<<grid, 32 * WROWS, 0, st>>>(a, h, h_f32, res, res_f32, gate);       \
        return true;
        LX2V_NORM_G(1) LX2V_NORM_G(2) LX2V_NORM_G(3) LX2V_NORM_G(4) LX2V_NORM_G(6) LX2V_NORM_G(8) LX2V_NORM_G(12)
#undef LX2V_NORM_G
        default: return false;
    }
}
static bool head_split_warp_launch(const HeadSplitArgs &a, cudaStream_t st) {
    const int d = a.heads * a.head_dim;
    if (a.src_f32 || d % 256 != 0 || a.head_dim % 8 != 0 || a.src_stride % 8 != 0 || a.col_off % 8 != 0)
        return false;
    const unsigned grid = (unsigned)((a.rows + WROWS - 1) / WROWS);
    switch (d / 256) {
#define LX2V_HS_G(G)                                                   \
    case G:                                                            \
        head_split_warp_kernel<G><<<grid, 32 * WROWS, 0, st>>>(a);     \
        return true;
        LX2V_HS_G(1) LX2V_HS_G(2) LX2V_HS_G(3) LX2V_HS_G(4) LX2V_HS_G(6) LX2V_HS_G(8) LX2V_HS_G(12)
#undef LX2V_HS_G
        default: return false;
    }
}

cudaError_t layer_norm_launch(const NormArgs &a, cudaStream_t st) {
    if (a.rows == 0) return cudaSuccess;
    if (norm_warp_launch<false>(a, nullptr, 0, nullptr, 0, -1, st)) return cudaGetLastError();
    if (vec_ok(a.dim)) {
        norm_vec_kernel<false><<<(unsigned)a.rows, a.dim / 8, 0, st>>>(a, nullptr, 0, nullptr, 0, -1);
        return cudaGetLastError();
    }
    layer_norm_kernel<<<(unsigned)a.rows, ROW_THREADS, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t residual_norm_launch(const NormArgs &a, void *h, int h_f32, const void *res, int res_f32, int gate,
                                 cudaStream_t st) {
    if (a.rows == 0) return cudaSuccess;
    if (norm_warp_launch<true>(a, h, h_f32, res, res_f32, gate, st)) return cudaGetLastError();
    if (vec_ok(a.dim)) {
        norm_vec_kernel<true><<<(unsigned)a.rows, a.dim / 8, 0, st>>>(a, h, h_f32, res, res_f32, gate);
        return cudaGetLastError();
    }
    residual_norm_kernel<<<(unsigned)a.rows, ROW_THREADS, 0, st>>>(a, h, h_f32, res, res_f32, gate);
    return cudaGetLastError();
}

cudaError_t head_split_launch(const HeadSplitArgs &a, cudaStream_t st) {
    if (a.rows == 0) return cudaSuccess;
    if (head_split_warp_launch(a, st)) return cudaGetLastError();
    const int d = a.heads * a.head_dim;
    // 8 values a thread never straddle a head; src rows, the column offset and
    // the RoPE rows stay 16-byte aligned
    if (vec_ok(d) && a.head_dim % 8 == 0 && a.src_stride % 8 == 0 && a.col_off % 8 == 0) {
        head_split_vec_kernel<<<(unsigned)a.rows, d / 8, 0, st>>>(a);
        return cudaGetLastError();
    }
    head_split_kernel<<<(unsigned)a.rows, ROW_THREADS, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t row_sumsq_launch(const void *src, int src_f32, int64_t rows, int64_t stride, int64_t col_off, int width,
                             float *out, cudaStream_t st) {
    if (rows == 0) return cudaSuccess;
    row_sumsq_kernel<<<(unsigned)rows, ROW_THREADS, 0, st>>>(src, src_f32, stride, col_off, width, out);
    return cudaGetLastError();
}

cudaError_t patchify_launch(const void *src, int src_f32, void *dst, int dst_f32, int c, int t, int h, int w, int p,
                            int to_tokens, cudaStream_t st) {
    const int64_t total = (int64_t)t * (h / p) * (w / p) * c * p * p;
    if (total == 0) return cudaSuccess;
    patchify_kernel<<<grid_elems(total), 256, 0, st>>>(src, src_f32, dst, dst_f32, c, t, h, w, p, to_tokens);
    return cudaGetLastError();
}

cudaError_t dmd_step_launch(void *x, int x_f32, const void *v, int v_f32, const void *noise, int n_f32, float sigma_t,
                            float sigma_next, int64_t n, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    dmd_step_kernel<<<grid_elems(n), 256, 0, st>>>(x, x_f32, v, v_f32, noise, n_f32, sigma_t, sigma_next, n);
    return cudaGetLastError();
}

}  // namespace lx2v
