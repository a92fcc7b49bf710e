// peer.cu — tensor parallelism over NVLink peer memory: a barrier between the
// ranks of a group and the reduce-scatter / residual / norm / all-gather
// step that follows each row-split linear of a DiT block.
//
// The reference runs a block on one device (crates/lightx2v-model/src/
// dit.rs:569-782): after out1, out2 and FFN2 it adds the (gated) product into
// the residual stream h and normalises h for the next linear
// (residual_norm, crates/lightx2v-cpu/src/lib.rs:364-392; the FFN's
// gate_residual :394-404 followed by the next block's layer_norm :328-362).
// Split over P ranks, each row-split linear leaves every rank with a partial
// product of all M rows. Each rank owns a contiguous range of rows; one
// kernel per rank then, for each owned row:
//   - reads that row of every rank's partial over NVLink (peer loads of
//     buffers shared by CUDA IPC) and adds them in rank order, in f32
//     (the reduce-scatter);
//   - adds the sum (times the gate) into its own rows of h;
//   - normalises the row (affine or modulated LayerNorm);
//   - stores the normalised row into every rank's activation buffer (the
//     all-gather), so the next column-split linear finds all M rows locally.
// Bytes per rank per step: (P-1)/P of a partial read and of the activation
// written over NVLink, the same as an all-reduce of the partial, with the
// row-wise work split P ways instead of repeated on every rank.
//
// peer_barrier_kernel orders these steps across the ranks: each rank stores
// the barrier's epoch into its slot of every rank's flag array (system-scope
// release after a system-scope fence, so the rank's earlier writes to peer
// memory are visible first) and waits until its own array holds the epoch
// from every rank (acquire loads). The wait is bounded: on expiry it records
// an error word that the next lx2v_sync reports, and returns.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include "peer.h"
#include "ptx.cuh"

namespace lx2v {

namespace {

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__global__ void peer_barrier_kernel(PeerFlags f, int world, int rank, unsigned epoch, int *err, uint64_t limit_ns) {
    if (threadIdx.x != 0) return;
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    for (int r = 0; r < world; ++r) st_release_sys(f.flags[r] + rank, epoch);
    const uint64_t t0 = globaltimer_ns();
    for (int r = 0; r < world; ++r) {
        for (;;) {
            if ((int)(ld_acquire_sys(f.flags[rank] + r) - epoch) >= 0) break;
            if (globaltimer_ns() - t0 > limit_ns) {
                raise_error(err, ERR_WAIT_TIMEOUT);
                return;
            }
            __nanosleep(64);
        }
    }
}

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

__device__ __forceinline__ uint32_t pack2(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// Sum over the CTA; every thread gets the total. `red` holds one float per warp.
__device__ __forceinline__ float cta_sum(float v, float *red) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    return t;
}

// One CTA per owned row, eight consecutive values per thread.
__global__ void __launch_bounds__(1024) tp_reduce_norm_kernel(TpNormArgs a) {
    __shared__ float red[32];
    const int64_t r = a.row0 + blockIdx.x;
    const int j0 = threadIdx.x * 8;
    const bool act = j0 < a.dim;
    const int64_t i0 = r * a.dim + j0;
    float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (act) {
        float hv[8];
        ld8(a.h, 1, i0, hv);
        if (a.n_parts > 0) {
            float s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (int p = 0; p < a.n_parts; ++p) {  // rank order: the same sum on every run
                float t[8];
                ld8(a.parts[p], a.parts_f32, i0, t);
#pragma unroll
                for (int k = 0; k < 8; ++k) s[k] += t[k];
            }
            float g[8] = {1, 1, 1, 1, 1, 1, 1, 1};
            if (a.gate >= 0) ld8(a.gmods, a.gmods_f32, (int64_t)a.gate * a.dim + j0, g);
#pragma unroll
            for (int k = 0; k < 8; ++k) hv[k] += s[k] * g[k];
            float *hp = reinterpret_cast<float *>(a.h) + i0;
            *reinterpret_cast<float4 *>(hp) = make_float4(hv[0], hv[1], hv[2], hv[3]);
            *reinterpret_cast<float4 *>(hp + 4) = make_float4(hv[4], hv[5], hv[6], hv[7]);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = hv[k];
    }
    float s1 = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) s1 += v[k];
    const float mean = cta_sum(s1, red) / (float)a.dim;
    float s2 = 0.0f;
    if (act) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float c = v[k] - mean;
            s2 += c * c;
        }
    }
    const float var = cta_sum(s2, red) / (float)a.dim;
    const float inv = 1.0f / sqrtf(var + a.eps);
    if (!act) return;
    float m1[8], m2[8];
    if (a.kind == 0) {
        ld8(a.w, a.w_f32, j0, m1);
        ld8(a.b, a.b_f32, j0, m2);
    } else {
        ld8(a.nmods, a.nmods_f32, (int64_t)a.scale * a.dim + j0, m1);
        ld8(a.nmods, a.nmods_f32, (int64_t)a.shift * a.dim + j0, m2);
#pragma unroll
        for (int k = 0; k < 8; ++k) m1[k] += 1.0f;
    }
    float o[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) o[k] = (v[k] - mean) * inv * m1[k] + m2[k];
    const uint4 packed = make_uint4(pack2(o[0], o[1]), pack2(o[2], o[3]), pack2(o[4], o[5]), pack2(o[6], o[7]));
    for (int p = 0; p < a.n_outs; ++p) {  // this rank's rows into every rank's buffer
        if (a.out_f32) {
            float *d = reinterpret_cast<float *>(a.outs[p]) + i0;
            *reinterpret_cast<float4 *>(d) = make_float4(o[0], o[1], o[2], o[3]);
            *reinterpret_cast<float4 *>(d + 4) = make_float4(o[4], o[5], o[6], o[7]);
        } else {
            *reinterpret_cast<uint4 *>(reinterpret_cast<__nv_bfloat16 *>(a.outs[p]) + i0) = packed;
        }
    }
}

// One warp per row: the sum of squares of its columns, into every rank's slot.
__global__ void __launch_bounds__(256) row_sumsq_peers_kernel(PeerRowSums a) {
    const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= a.rows) return;
    const int64_t base = r * a.stride + a.col_off;
    float s = 0.0f;
    if (!a.src_f32 && a.width % 8 == 0 && base % 8 == 0) {
        for (int j = lane * 8; j < a.width; j += 256) {
            float v[8];
            ld8(a.src, 0, base + j, v);
#pragma unroll
            for (int k = 0; k < 8; ++k) s += v[k] * v[k];
        }
    } else {
        for (int j = lane; j < a.width; j += 32) {
            const float v = a.src_f32 ? reinterpret_cast<const float *>(a.src)[base + j]
                                      : __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(a.src)[base + j]);
            s += v * v;
        }
    }
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
    if (lane < a.n_outs) a.outs[lane][a.slot + r] = s;
}

}  // namespace

cudaError_t row_sumsq_peers_launch(const PeerRowSums &a, cudaStream_t st) {
    row_sumsq_peers_kernel<<<(unsigned)((a.rows + 7) / 8), 256, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t peer_barrier_launch(const PeerFlags &f, int world, int rank, unsigned epoch, int *err, uint64_t limit_ns,
                                cudaStream_t st) {
    peer_barrier_kernel<<<1, 32, 0, st>>>(f, world, rank, epoch, err, limit_ns);
    return cudaGetLastError();
}

bool tp_reduce_norm_supported(int dim) { return dim > 0 && dim % 8 == 0 && dim <= 8 * 1024; }

cudaError_t tp_reduce_norm_launch(const TpNormArgs &a, cudaStream_t st) {
    if (a.row1 <= a.row0) return cudaSuccess;
    const int threads = ((a.dim / 8 + 31) / 32) * 32;
    tp_reduce_norm_kernel<<<(unsigned)(a.row1 - a.row0), threads, 0, st>>>(a);
    return cudaGetLastError();
}

}  // namespace lx2v
