// gemv.cu — the quantized linear for a few tokens (M <= 16): bandwidth-bound.
//
// Same computation as Backend::linear (crates/lightx2v-core/src/backend.rs:
// 199-212; CPU reference crates/lightx2v-cpu/src/lib.rs:296-326) with the same
// operand rounding as the tensor-core kernels (exact dequantisation rounded to
// bf16, activations bf16, f32 accumulation), for the regime where the weight
// stream dominates: every weight byte is read once, 16 bytes per thread per
// load, and decoded in registers straight into mma.sync B fragments.
//
// Work split: a CTA of 8 warps owns 64 weight rows (8 per warp, the MMA's N)
// and one k-range (split-K when there are too few row tiles to fill the GPU).
// The MMA's M = 16 token rows (x rows beyond M are zero); x's k-range is
// staged in shared memory once per CTA.
//
// k permutation: in mma.m16n8k16 the thread with c = lane % 4 holds the B
// values at k positions {2c, 2c+1, 2c+8, 2c+9} of a 16-wide step. Thread c
// loads 16 (Q4: 32) contiguous codes of its row, k = kc + c*VT + j, and step
// s uses its values j = 4s..4s+3 at those positions; the A fragment (x) of
// the threads with the same c reads x at the same four k, so every k of the
// chunk meets its own x exactly once and the dot products are unchanged.
//
// Split-K partials go to a workspace; the last CTA of a row tile (atomic
// arrival count, reset by that CTA) adds them in split order, so results do
// not depend on CTA timing.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <cstring>
#include "gemm_common.cuh"  // decoders, GELU

namespace lx2v {

namespace {

constexpr int GV_WARPS = 8;
constexpr int GV_ROWS = 8 * GV_WARPS;  // weight rows per CTA
constexpr int GV_THREADS = 32 * GV_WARPS;

template <int FMT>
struct GvFmt {
    static constexpr int UNITS = FMT == FMT_Q4 ? 2 : 1;  // 16-value units per thread per chunk
    static constexpr int VT = 16 * UNITS;                // values per thread per chunk
    static constexpr int KC = 4 * VT;                    // k per warp chunk
    static constexpr int STEPS = VT / 4;                 // mma k-steps per chunk
};

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float ld_elem(const void *p, int f32, int64_t i) {
    return f32 ? reinterpret_cast<const float *>(p)[i] : __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[i]);
}

// Everything one thread reads from HBM for one chunk: its codes (16 bytes;
// 32 for bf16 weights), the scale word of their group and, for FP8, the
// block flag. All of it is loaded up front so every load of the thread's
// k-range is in flight at once.
template <int FMT>
struct GvChunk {
    uint4 a, b;
    uint32_t side;  // f32 scale (Q8/FP8) or half2 (scale, zero) (Q4)
    uint32_t mode;  // FP8 block flag
};

template <int FMT>
__device__ __forceinline__ void gv_load(const LinearArgs &a, int n, int k, GvChunk<FMT> &r) {
    r.a = make_uint4(0, 0, 0, 0);
    r.b = make_uint4(0, 0, 0, 0);
    r.side = 0;
    r.mode = 0;
    if (n >= a.N) return;
    if (FMT == FMT_Q4) {
        r.a = __ldg(reinterpret_cast<const uint4 *>(a.codes + ((int64_t)n * a.K + k) / 2));
        r.side = __ldg(a.sz_t + (int64_t)(k / a.group) * a.N + n);
    } else if (FMT == FMT_BF16) {
        const uint4 *p = reinterpret_cast<const uint4 *>(a.codes + ((int64_t)n * a.K + k) * 2);
        r.a = __ldg(p);
        r.b = __ldg(p + 1);
    } else {
        r.a = __ldg(reinterpret_cast<const uint4 *>(a.codes + (int64_t)n * a.K + k));
        r.side = __float_as_uint(__ldg(a.scales_t + (int64_t)(k / a.group) * a.N + n));
        if (FMT == FMT_FP8) r.mode = __ldg(a.flags + (int64_t)(k / 32) * a.N + n);
    }
}

// Decode one thread's chunk to bf16 pairs: out[8u + i] = values
// (16u + 2i, 16u + 2i + 1). A thread's chunk never straddles a scale group
// or an FP8 flag block (gemv_supported).
template <int FMT>
__device__ __forceinline__ void gv_decode(const GvChunk<FMT> &r, uint32_t (&out)[8 * GvFmt<FMT>::UNITS]) {
#pragma unroll
    for (int u = 0; u < GvFmt<FMT>::UNITS; ++u) {
        uint32_t o[8];
        if (FMT == FMT_BF16) {
            unit_to_bf16<FMT_BF16>(r.a, r.b, 0.0f, 0.0f, 0, o);
        } else if (FMT == FMT_Q4) {
            float sc, z;
            q4_scale_zero(r.side, sc, z);
            const uint4 r4 = u == 0 ? make_uint4(r.a.x, r.a.y, 0, 0) : make_uint4(r.a.z, r.a.w, 0, 0);
            unit_to_bf16<FMT_Q4>(r4, r4, sc, z, 0, o);
        } else {
            unit_to_bf16<FMT>(r.a, r.a, __uint_as_float(r.side), 0.0f, (int)r.mode, o);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) out[8 * u + i] = o[i];
    }
}

constexpr int GV_MAXCH = 8;  // chunks per thread (its whole k-range, loaded at once)

template <int FMT>
__global__ void __launch_bounds__(GV_THREADS) gemv_kernel(LinearArgs a, int splits, int kchunks_per_split,
                                                         float *partials, int *arrivals) {
    using F = GvFmt<FMT>;
    extern __shared__ __align__(16) uint8_t gv_smem[];
    const int tile = blockIdx.x / splits, split = blockIdx.x % splits;
    const int n_chunks = a.K / F::KC;
    const int c_begin = split * kchunks_per_split;
    const int nch = min(n_chunks - c_begin, kchunks_per_split);  // <= GV_MAXCH
    const int k_begin = c_begin * F::KC;
    const int kext = nch * F::KC;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, c = lane & 3;
    const int n_warp = tile * GV_ROWS + warp * 8;  // first of this warp's 8 rows
    const int n = n_warp + g;                      // this thread's B row

    // Launched as a programmatic dependent of the previous kernel: the next
    // kernel may launch as soon as every CTA of this one has started, and
    // this one's weight loads (immutable, nothing earlier in the stream
    // writes them) are in flight before it waits for the previous kernel.
    griddep_launch_dependents();

    // 1. issue every weight load of this thread's k-range
    GvChunk<FMT> ck[GV_MAXCH];
#pragma unroll
    for (int j = 0; j < GV_MAXCH; ++j)
        if (j < nch) gv_load<FMT>(a, n, k_begin + j * F::KC + c * F::VT, ck[j]);

    // everything below reads x or writes y / partials / arrival counters,
    // which earlier kernels in the stream may still use
    griddep_wait();

    // 2. meanwhile stage x rows (16, zero beyond M) of the k-range as bf16,
    //    row stride kext + 8, 8 values per thread and step
    const int xs_stride = kext + 8;
    __nv_bfloat16 *xs = reinterpret_cast<__nv_bfloat16 *>(gv_smem);
    const int per_row = kext / 8;
    for (int e = threadIdx.x; e < 16 * per_row; e += GV_THREADS) {
        const int r = e / per_row, kk = 8 * (e - r * per_row);
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < a.M) {
            const int64_t base = ((int64_t)a.x_row + r) * a.K + k_begin + kk;
            if (a.x_f32) {
                const float4 f0 = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(a.x) + base);
                const float4 f1 = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(a.x) + base + 4);
                v.x = pack_bf16x2(f0.x, f0.y); v.y = pack_bf16x2(f0.z, f0.w);
                v.z = pack_bf16x2(f1.x, f1.y); v.w = pack_bf16x2(f1.z, f1.w);
            } else {
                v = *reinterpret_cast<const uint4 *>(reinterpret_cast<const __nv_bfloat16 *>(a.x) + base);
            }
        }
        *reinterpret_cast<uint4 *>(xs + r * xs_stride + kk) = v;
    }
    __syncthreads();

    // 3. decode and multiply, chunk by chunk
    float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const uint32_t xrow0 = (uint32_t)__cvta_generic_to_shared(xs + g * xs_stride);
    const uint32_t xrow1 = (uint32_t)__cvta_generic_to_shared(xs + (g + 8) * xs_stride);
#pragma unroll
    for (int j = 0; j < GV_MAXCH; ++j) {
        if (j >= nch) break;
        uint32_t w[8 * F::UNITS];
        gv_decode<FMT>(ck[j], w);
        const uint32_t xoff = (uint32_t)((j * F::KC + c * F::VT) * 2);
#pragma unroll
        for (int s = 0; s < F::STEPS; ++s) {
            uint32_t x00, x01, x10, x11;
            asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(x00), "=r"(x01) : "r"(xrow0 + xoff + 8 * s));
            asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(x10), "=r"(x11) : "r"(xrow1 + xoff + 8 * s));
            mma_bf16_16816(d, x00, x10, x01, x11, w[2 * s], w[2 * s + 1]);
        }
    }

    // C fragment: d0, d1 = token g, rows n_warp + 2c, +1; d2, d3 = token g + 8.
    const int nc = n_warp + 2 * c;
    if (splits > 1) {
        float *mine = partials + (int64_t)blockIdx.x * (16 * GV_ROWS);
        const int col = warp * 8 + 2 * c;
        __stcg(reinterpret_cast<float2 *>(mine + g * GV_ROWS + col), make_float2(d[0], d[1]));
        __stcg(reinterpret_cast<float2 *>(mine + (g + 8) * GV_ROWS + col), make_float2(d[2], d[3]));
        // the CTA's partial stores, then one GPU-scope fence (cumulative over
        // the stores the barrier ordered before it) and the arrival
        __syncthreads();
        __shared__ int last;
        if (threadIdx.x == 0) {
            __threadfence();
            last = atomicAdd(arrivals + tile, 1) == splits - 1;
            if (last) __threadfence();  // the other CTAs' partials are visible below
        }
        __syncthreads();
        if (!last) return;
        float t[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int sp = 0; sp < splits; ++sp) {
            const float *p = partials + (int64_t)(tile * splits + sp) * (16 * GV_ROWS);
            const float2 u0 = __ldcg(reinterpret_cast<const float2 *>(p + g * GV_ROWS + col));
            const float2 u1 = __ldcg(reinterpret_cast<const float2 *>(p + (g + 8) * GV_ROWS + col));
            t[0] += u0.x; t[1] += u0.y; t[2] += u1.x; t[3] += u1.y;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) d[i] = t[i];
        if (threadIdx.x == 0) arrivals[tile] = 0;  // ready for the next launch
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int tok = g + 8 * h;
        if (tok >= a.M) continue;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int nn = nc + j;
            if (nn >= a.N) continue;
            float v = d[2 * h + j];
            if (a.bias) v += ld_elem(a.bias, a.bias_f32, nn);
            if (a.act == 1) v = gelu2(make_float2(v, v)).x;
            const int64_t yi = ((int64_t)a.y_row + tok) * a.N + nn;
            if (a.gate) v = ld_elem(a.y, a.y_f32, yi) + v * ld_elem(a.gate, a.gate_f32, nn);
            if (a.y_f32) reinterpret_cast<float *>(a.y)[yi] = v;
            else reinterpret_cast<__nv_bfloat16 *>(a.y)[yi] = __float2bfloat16_rn(v);
        }
    }
}

template <int FMT>
cudaError_t gemv_launch_t(const LinearArgs &a, int num_sms, float *partials, int *arrivals, size_t ws_floats,
                          cudaStream_t st) {
    using F = GvFmt<FMT>;
    const int tiles = (a.N + GV_ROWS - 1) / GV_ROWS;
    const int n_chunks = a.K / F::KC;
    // every split at most GV_MAXCH chunks (a thread loads its whole range at
    // once); more splits only while the GPU has fewer than two CTAs per SM
    int splits = (n_chunks + GV_MAXCH - 1) / GV_MAXCH;
    while (tiles * splits < 2 * num_sms && n_chunks / (splits + 1) >= 2) ++splits;
    const int per = (n_chunks + splits - 1) / splits;
    splits = (n_chunks + per - 1) / per;
    if (splits > 1 && (size_t)tiles * splits * 16 * GV_ROWS > ws_floats) return cudaErrorInvalidValue;
    const size_t smem = (size_t)16 * (per * F::KC + 8) * 2;
    auto kern = gemv_kernel<FMT>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof cfg);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(tiles * splits);
    cfg.blockDim = dim3(GV_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a, splits, per, partials, arrivals);
}

}  // namespace

bool gemv_supported(const LinearArgs &a) {
    if (a.M < 1 || a.M > 16 || a.N < 1) return false;
    switch (a.fmt) {
        case FMT_Q4:  // this kernel, or gemv_q4.cu's for groups of 64k
            return (a.K % GvFmt<FMT_Q4>::KC == 0 && a.group % 32 == 0) ||
                   (a.K % 64 == 0 && a.group % 64 == 0 && a.K % a.group == 0 && a.K <= 49152);
        case FMT_Q8:
        case FMT_FP8: return a.K % 64 == 0 && a.group % 16 == 0;
        case FMT_NVFP4: return false;  // two-pass or generic kernel
        default: return a.K % 64 == 0;
    }
}

// partials: at least gemv_workspace_floats(N, K, num_sms) floats; arrivals:
// ceil(N / 64) ints, zero before the first launch (kernels leave them zero).
size_t gemv_workspace_floats(int N, int K, int num_sms) {
    // the largest split count gemv_launch_t picks for this shape (Q8/FP8/bf16
    // chunks are the narrowest, so they need the most splits)
    const int tiles = (N + GV_ROWS - 1) / GV_ROWS;
    const int n_chunks = K / 64;
    int splits = (n_chunks + GV_MAXCH - 1) / GV_MAXCH;
    while (tiles * splits < 2 * num_sms && n_chunks / (splits + 1) >= 2) ++splits;
    return (size_t)tiles * (splits < 1 ? 1 : splits) * 16 * GV_ROWS;
}

cudaError_t linear_gemv_launch(const LinearArgs &a, int num_sms, cudaStream_t st, float *partials, int *arrivals,
                               size_t ws_floats) {
    switch (a.fmt) {
        case FMT_Q8: return gemv_launch_t<FMT_Q8>(a, num_sms, partials, arrivals, ws_floats, st);
        case FMT_Q4:
            if (gemv_q4_supported(a, num_sms)) return gemv_q4_launch(a, num_sms, st);
            return gemv_launch_t<FMT_Q4>(a, num_sms, partials, arrivals, ws_floats, st);
        case FMT_FP8: return gemv_launch_t<FMT_FP8>(a, num_sms, partials, arrivals, ws_floats, st);
        default: return gemv_launch_t<FMT_BF16>(a, num_sms, partials, arrivals, ws_floats, st);
    }
}

}  // namespace lx2v
