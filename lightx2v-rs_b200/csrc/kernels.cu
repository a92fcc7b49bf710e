// kernels.cu — the non-tensor-core kernels of the backend:
//   convert          f32 <-> bf16 element conversion (upload / download / copy)
//   gate_residual    Backend::gate_residual, crates/lightx2v-cpu/src/lib.rs:394-404
//   dequant_f32      bit-exact weight decode (test hook for quant.rs dequantize)
//   dequant_bf16     first pass of the two-pass linear: the bf16 weight operand
//   linear_simt      Backend::linear for shapes the tensor-core kernel does not
//                    take (K not a multiple of 16, odd groups, tiny M, f32 x).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <cstring>
#include "dequant.cuh"
#include "gemm.h"
#include "ptx.cuh"

namespace lx2v {

__device__ __forceinline__ float load_elem(const void *p, int f32, int64_t i) {
    return f32 ? reinterpret_cast<const float *>(p)[i]
               : __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[i]);
}
__device__ __forceinline__ void store_elem(void *p, int f32, int64_t i, float v) {
    if (f32) reinterpret_cast<float *>(p)[i] = v;
    else reinterpret_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v);
}

static int grid_for(size_t n, int threads) {
    size_t g = (n + threads - 1) / threads;
    if (g > 148 * 32) g = 148 * 32;
    if (g < 1) g = 1;
    return (int)g;
}

// ---- convert --------------------------------------------------------------
__global__ void convert_kernel(const void *src, int src_f32, void *dst, int dst_f32, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        store_elem(dst, dst_f32, (int64_t)i, load_elem(src, src_f32, (int64_t)i));
}

cudaError_t convert_launch(const void *src, int src_f32, void *dst, int dst_f32, size_t n,
                           cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    convert_kernel<<<grid_for(n, 256), 256, 0, st>>>(src, src_f32, dst, dst_f32, n);
    return cudaGetLastError();
}

// ---- gate_residual ---------------------------------------------------------
// h[r, j] += a[r, j] * gate[j]   (gate = mods + gate_slot * dim)
__global__ void gate_residual_kernel(void *h, int h_f32, const void *a, int a_f32, const void *gate,
                                     int gate_f32, size_t rows, size_t dim) {
    const size_t n = rows * dim;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t j = i % dim;
        const float v = load_elem(h, h_f32, (int64_t)i) +
                        load_elem(a, a_f32, (int64_t)i) * load_elem(gate, gate_f32, (int64_t)j);
        store_elem(h, h_f32, (int64_t)i, v);
    }
}

cudaError_t gate_residual_launch(void *h, int h_f32, const void *a, int a_f32, const void *gate,
                                 int gate_f32, size_t rows, size_t dim, cudaStream_t st) {
    const size_t n = rows * dim;
    if (n == 0) return cudaSuccess;
    gate_residual_kernel<<<grid_for(n, 256), 256, 0, st>>>(h, h_f32, a, a_f32, gate, gate_f32, rows, dim);
    return cudaGetLastError();
}

// ---- dequant hook ------------------------------------------------------------
// Unit path: the same decode functions the GEMM's dequant warps run, with
// the same fast/reference split for FP8.
template <int FMT>
__global__ void dequant_units_kernel(WeightView w, float *out) {
    const int units_per_row = w.k / 16;
    const int64_t total = (int64_t)w.n * units_per_row;
    for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < total; u += (int64_t)gridDim.x * blockDim.x) {
        const int n = (int)(u / units_per_row), k0 = (int)(u % units_per_row) * 16;
        const int64_t base = (int64_t)n * w.k + k0;
        const int64_t g = k0 / w.group;
        float v[16];
        if (FMT == FMT_Q4) {
            const uint2 raw = *reinterpret_cast<const uint2 *>(w.codes + base / 2);
            float s, z;
            q4_scale_zero(w.sz_t[g * w.n + n], s, z);
            unit_to_f32<FMT_Q4>(make_uint4(raw.x, raw.y, 0, 0), s, z, 0, v);
        } else if (FMT == FMT_NVFP4) {
            const uint2 raw = *reinterpret_cast<const uint2 *>(w.codes + base / 2);
            unit_to_f32<FMT_NVFP4>(make_uint4(raw.x, raw.y, 0, 0), w.scales_t[g * w.n + n], 0.0f, 0, v);
        } else if (FMT == FMT_BF16) {
            const __nv_bfloat16 *p = reinterpret_cast<const __nv_bfloat16 *>(w.codes) + base;
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = __bfloat162float(p[i]);
        } else {
            const uint4 raw = *reinterpret_cast<const uint4 *>(w.codes + base);
            const int mode = FMT == FMT_FP8 ? w.flags[(int64_t)(k0 / 32) * w.n + n] : 0;
            unit_to_f32<FMT>(raw, w.scales_t[g * w.n + n], 0.0f, mode, v);
        }
        float4 *o = reinterpret_cast<float4 *>(out + base);
#pragma unroll
        for (int i = 0; i < 4; ++i) o[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    }
}
// Element path for shapes outside the unit path.
__global__ void dequant_elems_kernel(WeightView w, float *out) {
    const int64_t total = (int64_t)w.n * w.k;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = dq_elem(w, i / w.k, i % w.k);
}

// ---- dequant to bf16 (first pass of the two-pass linear) --------------------------
// Row-major bf16 copy of the weight, [N][K], each value the decoded weight
// rounded to nearest-even: the same bf16 operand that the dequant warps of the
// one-pass kernels write into TMEM (unit_to_bf16, with the FP8 blocks' flag
// choosing the hardware, fixed-up or reference decode), so both kinds of
// kernel multiply identical operands. Thread = one 16-value unit; consecutive
// threads take consecutive units of a row (16-byte code loads, 32-byte stores).
// Launched as a programmatic dependent of the previous kernel in the stream:
// it reads only the weight, so it runs beside that kernel's last tiles, lets
// the GEMM that consumes it launch (and set up) right away, and before
// exiting waits for the previous kernel, so that whatever follows this pass
// in the stream also follows everything before it.
template <int FMT>
__global__ void __launch_bounds__(256) dequant_bf16_kernel(WeightView w, __nv_bfloat16 *out) {
    griddep_launch_dependents();
    const int units_per_row = w.k / 16;
    const int64_t total = (int64_t)w.n * units_per_row;
    for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < total; u += (int64_t)gridDim.x * blockDim.x) {
        const int n = (int)(u / units_per_row), k0 = (int)(u % units_per_row) * 16;
        const int64_t base = (int64_t)n * w.k + k0;
        const int64_t g = k0 / w.group;
        uint32_t o[8];
        if (FMT == FMT_Q4) {
            const uint2 raw = __ldg(reinterpret_cast<const uint2 *>(w.codes + base / 2));
            float s, z;
            q4_scale_zero(__ldg(w.sz_t + g * w.n + n), s, z);
            unit_to_bf16<FMT_Q4>(make_uint4(raw.x, raw.y, 0, 0), make_uint4(0, 0, 0, 0), s, z, 0, o);
        } else if (FMT == FMT_NVFP4) {
            const uint2 raw = __ldg(reinterpret_cast<const uint2 *>(w.codes + base / 2));
            unit_to_bf16<FMT_NVFP4>(make_uint4(raw.x, raw.y, 0, 0), make_uint4(0, 0, 0, 0),
                                    __ldg(w.scales_t + g * w.n + n), 0.0f, 0, o);
        } else {
            const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(w.codes + base));
            const int mode = FMT == FMT_FP8 ? __ldg(w.flags + (int64_t)(k0 / 32) * w.n + n) : 0;
            unit_to_bf16<FMT>(raw, raw, __ldg(w.scales_t + g * w.n + n), 0.0f, mode, o);
        }
        uint4 *dst = reinterpret_cast<uint4 *>(out + base);
        dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
        dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
    }
    griddep_wait();
}

cudaError_t dequant_bf16_launch(int fmt, const uint8_t *codes, const float *scales_t, const uint32_t *sz_t,
                                const uint8_t *flags, int N, int K, int group, __nv_bfloat16 *out,
                                cudaStream_t st) {
    WeightView w{fmt, N, K, group, codes, scales_t, sz_t, flags};
    if ((size_t)N * K == 0) return cudaSuccess;
    if (fmt == FMT_BF16 || !unit_path_ok(fmt, K, group)) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof cfg);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(grid_for((size_t)N * K / 16, 256));
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    switch (fmt) {
        case FMT_Q8: return cudaLaunchKernelEx(&cfg, dequant_bf16_kernel<FMT_Q8>, w, out);
        case FMT_Q4: return cudaLaunchKernelEx(&cfg, dequant_bf16_kernel<FMT_Q4>, w, out);
        case FMT_NVFP4: return cudaLaunchKernelEx(&cfg, dequant_bf16_kernel<FMT_NVFP4>, w, out);
        default: return cudaLaunchKernelEx(&cfg, dequant_bf16_kernel<FMT_FP8>, w, out);
    }
}

cudaError_t dequant_f32_launch(int fmt, const uint8_t *codes, const float *scales_t,
                               const uint32_t *sz_t, const uint8_t *flags, int N, int K, int group,
                               float *out, cudaStream_t st) {
    WeightView w{fmt, N, K, group, codes, scales_t, sz_t, flags};
    if ((size_t)N * K == 0) return cudaSuccess;
    if (unit_path_ok(fmt, K, group)) {
        const int g = grid_for((size_t)N * K / 16, 256);
        switch (fmt) {
            case FMT_Q8: dequant_units_kernel<FMT_Q8><<<g, 256, 0, st>>>(w, out); break;
            case FMT_Q4: dequant_units_kernel<FMT_Q4><<<g, 256, 0, st>>>(w, out); break;
            case FMT_FP8: dequant_units_kernel<FMT_FP8><<<g, 256, 0, st>>>(w, out); break;
            case FMT_NVFP4: dequant_units_kernel<FMT_NVFP4><<<g, 256, 0, st>>>(w, out); break;
            default: dequant_units_kernel<FMT_BF16><<<g, 256, 0, st>>>(w, out); break;
        }
    } else {
        dequant_elems_kernel<<<grid_for((size_t)N * K, 256), 256, 0, st>>>(w, out);
    }
    return cudaGetLastError();
}

// ---- generic CUDA-core linear ----------------------------------------------
// 64x64 output tile per 256-thread block, 4x4 outputs per thread, K step 16.
// Weights are the exact decoded value rounded to bf16 and activations are
// rounded to bf16, the same operand rounding as the tensor-core kernel.
__device__ __forceinline__ float round_bf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__global__ void __launch_bounds__(256) linear_simt_kernel(LinearArgs a) {
    __shared__ float xs[16][65];
    __shared__ float ws[16][65];
    WeightView w{a.fmt, a.N, a.K, a.group, a.codes, a.scales_t, a.sz_t, a.flags};
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < a.K; k0 += 16) {
        for (int e = threadIdx.x; e < 64 * 16; e += 256) {
            const int r = e / 16, kk = e % 16, gk = k0 + kk;
            float xv = 0.0f, wv = 0.0f;
            if (m0 + r < a.M && gk < a.K)
                xv = round_bf16(load_elem(a.x, a.x_f32, (a.x_row + m0 + r) * (int64_t)a.K + gk));
            if (n0 + r < a.N && gk < a.K) wv = round_bf16(dq_elem(w, n0 + r, gk));
            xs[kk][r] = xv;
            ws[kk][r] = wv;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {
            float xa[4], wb[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) { xa[i] = xs[kk][ty + 16 * i]; wb[i] = ws[kk][tx + 16 * i]; }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xa[i], wb[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + ty + 16 * i;
        if (m >= a.M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n0 + tx + 16 * j;
            if (n >= a.N) continue;
            float v = acc[i][j];
            if (a.bias) v += load_elem(a.bias, a.bias_f32, n);
            if (a.act == 1) {
                const float u = 0.7978845608028654f * (v + 0.044715f * v * v * v);
                v = v / (1.0f + expf(-2.0f * u));
            }
            const int64_t yi = (a.y_row + m) * (int64_t)a.N + n;
            if (a.gate) v = load_elem(a.y, a.y_f32, yi) + v * load_elem(a.gate, a.gate_f32, n);
            store_elem(a.y, a.y_f32, yi, v);
        }
    }
}

cudaError_t linear_simt_launch(const LinearArgs &a, cudaStream_t st) {
    if (a.M == 0 || a.N == 0) return cudaSuccess;
    dim3 grid((a.N + 63) / 64, (a.M + 63) / 64);
    linear_simt_kernel<<<grid, 256, 0, st>>>(a);
    return cudaGetLastError();
}

}  // namespace lx2v
