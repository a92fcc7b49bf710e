// gemv_q4.cu — the Q4 linear for a few tokens (M <= 16): the packed codes go
// into the tensor core as exact small integers and each scale group's affine
// map is applied to the group's partial dot products afterwards, in f32.
//
// Backend::linear (crates/lightx2v-core/src/backend.rs:199-212) on a Q4
// weight (crates/lightx2v-core/src/quant.rs:212-356; the CPU backend decodes
// w = (c - z) * s to f32 at upload, crates/lightx2v-cpu/src/lib.rs:259-284,
// then runs the dot product of :296-326). Grouping that dot product by scale
// group g of 64 (or a multiple of 64) k:
//
//     sum_k x[t,k] w[n,k] = sum_g s[n,g] * (sum_{k in g} x[t,k] c[n,k] - z[n,g] * X[t,g]),
//     X[t,g] = sum_{k in g} x[t,k].
//
// A code c enters mma.sync.m16n8k16 as the bf16 value 128 + c: the bit
// pattern 0x4300 | c, made for two codes at once by one lop3 on the packed
// nibbles. The MMA over a 64-wide chunk gives P = sum x (128 + c) (products of
// bf16 values are exact, sums in f32), and the chunk adds
// s * (P - (128 + z) X) to the output, with X the MMA of the same bf16 x
// values with an all-ones A. That is the reference's real number without rounding the weight to
// bf16 at all (every other CUDA path here multiplies bf16-rounded weights);
// x is bf16 as on every CUDA path (backend.rs:9-11). The decode is one shift
// and one lop3 per two codes, a tenth of the instructions of decoding each
// weight with the reference's roundings, which is what bounded the
// few-token kernel (gemv.cu).
//
// Work split. A warp owns one tile of 16 weight rows (the MMA's M; the
// tokens are the MMA's N = 8, two token tiles for M > 8) and a contiguous
// range of at most GQ_MAXC 64-wide k-chunks. A CTA of 8 warps holds `rt` row
// tiles x `ks` k-slices; a cluster of `cs` CTAs splits the k-range further.
// Every thread issues all of its weight loads (8 bytes of codes and one
// (scale, zero) word per row and chunk, rows g and g+8 of its tile) before
// waiting for the previous kernel in the stream (programmatic dependent
// launch), so the whole matrix is in flight at once. Then the CTA copies its
// k-range of x into shared memory (one bulk copy per token) and rewrites it in
// B-fragment order, with the sums X from the same fragments times an all-ones
// A. Partial sums meet in shared memory (the CTA's
// k-slices) and then in the cluster's distributed shared memory: each CTA
// owns a slice of the rows, receives every CTA's partial for them, adds them
// in rank order and runs the epilogue (bias, GELU, gated residual). Sums run
// in a fixed order, so results do not depend on timing; no global workspace.
//
// Fragment bookkeeping (lane = 4 g + t). In mma.m16n8k16 thread (g, t) holds
// A (weights) at rows g and g + 8 and at the k positions {2t, 2t+1, 2t+8,
// 2t+9} of the 16-wide step, and B (x) for token g at the same four k. The
// thread loads bytes [8t, 8t+8) of its two rows' 32-byte chunk: nibble i of
// the low word is k = 16t + i, of the high word k = 16t + 8 + i. lop3 on
// (word >> 4j) gives the bf16 pair (nibble j, nibble j + 4), so MMA 2h of the
// chunk takes the pairs j = 0, 1 of word h at positions (2t, 2t+1) and
// (2t+8, 2t+9), and MMA 2h + 1 the pairs j = 2, 3; the B fragments hold x at
// the same k, the pairs (x[16t + 8h + j], x[16t + 8h + j + 4]). Every k of the
// chunk meets its own x exactly once.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <cstring>
#include "gemm_common.cuh"

namespace lx2v {

namespace {

constexpr int GQ_WARPS = 8;
constexpr int GQ_THREADS = 32 * GQ_WARPS;
constexpr int GQ_MAXC = 12;  // 64-wide k-chunks per warp, all loaded at once
constexpr int GQ_MAXCS = 8;  // CTAs per cluster (portable limit)
constexpr uint32_t BF16X2_128 = 0x43004300u;
constexpr uint32_t NIB_LANES = 0x000F000Fu;

// bf16 pair (128 + nibble j, 128 + nibble j + 4) of a packed word
__device__ __forceinline__ uint32_t nib_pair(uint32_t w) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(w), "r"(NIB_LANES), "r"(BF16X2_128));  // (a & b) | c
    return r;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint2 ldg_stream_v2(const void *p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}
__device__ __forceinline__ uint32_t ldg_stream(const void *p) {
    uint32_t r;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
    return r;
}

__device__ __forceinline__ float ld_elem_q(const void *p, int f32, int64_t i) {
    return f32 ? reinterpret_cast<const float *>(p)[i] : __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[i]);
}

__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

// First chunk of k-slice s when C chunks are split into S slices.
__host__ __device__ __forceinline__ int slice_begin(int s, int S, int C) {
    return (int)(((long long)s * C) / S);
}

struct GqLayout {
    int xr_off, xr_stride, xs_off, xsum_off, red_off, recv_off, ep_off, bytes;
    int rows_per;  // rows of the CTA's group each cluster rank finalises
};

// Shared memory: the mbarrier; x rows as copied (MT * 8 tokens, bf16, the
// CTA's k-range, rows 16 bytes longer than a multiple of 128 so that 8 tokens
// x 4 lanes of 16-byte loads hit distinct banks); x again in B-fragment order
// (per chunk, token tile and half: 32 lanes x 16 bytes); the sums X; the
// warps' partials; the cluster receive buffer; bias and gate of the rows this
// CTA finalises.
__host__ __device__ inline GqLayout gq_layout(int mt, int cta_chunks, int rt, int cs) {
    GqLayout l;
    l.xr_off = 16;
    l.xr_stride = cta_chunks * 128 + 16;
    l.xs_off = l.xr_off + mt * 8 * l.xr_stride;
    l.xsum_off = l.xs_off + cta_chunks * mt * 1024;
    l.red_off = l.xsum_off + cta_chunks * 16 * 4;
    l.rows_per = (rt * 16 + cs - 1) / cs;
    l.recv_off = l.red_off + GQ_WARPS * 16 * 16 * 4;
    l.ep_off = l.recv_off + (cs > 1 ? cs * l.rows_per * 16 * 4 : 0);
    l.bytes = l.ep_off + 2 * rt * 16 * 4;
    return l;
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}

template <int MT>
__global__ void __launch_bounds__(GQ_THREADS, 2) gemv_q4_kernel(LinearArgs a, int rt, int ks, int cs, int max_cta_chunks) {
    extern __shared__ __align__(128) uint8_t gq_smem[];
    const int C = a.K / 64;
    const int S = ks * cs;
    const int crank = blockIdx.x;  // cluster dims (cs, 1, 1) and gridDim.x == cs
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int rti = warp % rt, ksi = warp / rt;
    const int row0 = (blockIdx.y * rt + rti) * 16;
    const int slice = crank * ks + ksi;
    const int cb = slice_begin(slice, S, C), nch = slice_begin(slice + 1, S, C) - cb;
    const int cta_lo = slice_begin(crank * ks, S, C), cta_hi = slice_begin((crank + 1) * ks, S, C);
    const int cta_chunks = cta_hi - cta_lo;
    const GqLayout L = gq_layout(MT, max_cta_chunks, rt, cs);
    uint64_t *bar = reinterpret_cast<uint64_t *>(gq_smem);
    const int R = rt * 16;
    const int group_row0 = blockIdx.y * R;
    const int rp = L.rows_per;
    const int my_lo = cs > 1 ? crank * rp : 0;
    const int my_rows = cs > 1 ? max(0, min(rp, R - my_lo)) : R;

    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    // The next kernel may start as soon as every CTA of this one runs; the
    // weights are immutable, so their loads go out before the wait below.
    griddep_launch_dependents();
    if (cs > 1) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");

    const int n_g = row0 + g, n_h = row0 + g + 8;
    const bool ok_g = n_g < a.N, ok_h = n_h < a.N;
    const int64_t rowb = a.K / 2;
    uint2 cg[GQ_MAXC], ch[GQ_MAXC];
    uint32_t sg[GQ_MAXC], sh[GQ_MAXC];
#pragma unroll
    for (int j = 0; j < GQ_MAXC; ++j) {
        cg[j] = ch[j] = make_uint2(0, 0);
        sg[j] = sh[j] = 0;
        if (j < nch) {
            const int c = cb + j;
            const int64_t gi = (int64_t)(c * 64 / a.group) * a.N;
            if (ok_g) {
                cg[j] = ldg_stream_v2(a.codes + n_g * rowb + c * 32 + 8 * t);
                sg[j] = ldg_stream(a.sz_t + gi + n_g);
            }
            if (ok_h) {
                ch[j] = ldg_stream_v2(a.codes + n_h * rowb + c * 32 + 8 * t);
                sh[j] = ldg_stream(a.sz_t + gi + n_h);
            }
        }
    }
    __syncthreads();  // the barrier's initialisation

    // x, bias, gate and y may still be in use by the previous kernel
    griddep_wait();

    // x rows of the CTA's k-range into shared memory: bf16 by bulk copies
    // (all in flight at once), f32 converted by the threads.
    const uint32_t xr_s = smem_u32(gq_smem + L.xr_off);
    const uint32_t row_bytes = (uint32_t)cta_chunks * 128;
    if (!a.x_f32) {
        if (threadIdx.x == 0) {
            mbar_arrive_expect_tx(bar, row_bytes * (uint32_t)a.M);
            for (int tok = 0; tok < a.M; ++tok) {
                const __nv_bfloat16 *src = reinterpret_cast<const __nv_bfloat16 *>(a.x) +
                                           (a.x_row + tok) * (int64_t)a.K + (int64_t)cta_lo * 64;
                bulk_g2s(xr_s + tok * L.xr_stride, src, row_bytes, smem_u32(bar));
            }
        }
    } else {
        const int pieces = cta_chunks * 8;  // 8 values each
        for (int e = threadIdx.x; e < a.M * pieces; e += GQ_THREADS) {
            const int tok = e / pieces, pc = e - tok * pieces;
            const float4 *p = reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(a.x) +
                                                               (a.x_row + tok) * (int64_t)a.K +
                                                               (int64_t)cta_lo * 64 + pc * 8);
            const float4 f0 = p[0], f1 = p[1];
            *reinterpret_cast<uint4 *>(gq_smem + L.xr_off + tok * L.xr_stride + pc * 16) =
                make_uint4(pack_bf16x2(f0.x, f0.y), pack_bf16x2(f0.z, f0.w), pack_bf16x2(f1.x, f1.y),
                           pack_bf16x2(f1.z, f1.w));
        }
    }
    // bias and gate of the rows this CTA finalises, while x is in flight
    float *ep = reinterpret_cast<float *>(gq_smem + L.ep_off);
    if (threadIdx.x < my_rows) {
        const int n = group_row0 + my_lo + threadIdx.x;
        ep[threadIdx.x] = a.bias && n < a.N ? ld_elem_q(a.bias, a.bias_f32, n) : 0.0f;
        ep[R + threadIdx.x] = a.gate && n < a.N ? ld_elem_q(a.gate, a.gate_f32, n) : 0.0f;
    }
    if (!a.x_f32) mbar_wait_bounded(bar, 0, a.err, a.wait_limit_ns);
    __syncthreads();
    const uint8_t *xr = gq_smem + L.xr_off;

    // x in B-fragment order and the sums X, one warp per (chunk, token
    // tile): lane (g, t) takes the 16 x values of token g at k = 16t.. of
    // the chunk and pairs them (x0,x4) (x1,x5) (x2,x6) (x3,x7) per 8 (the k of
    // MMA 2h and 2h + 1); X = the same fragments times an all-ones A, which
    // lands in the C layout (token 2t, 2t+1 on every row).
    const uint32_t ONES = 0x3F803F80u;  // bf16 pair (1, 1)
    uint4 *xs = reinterpret_cast<uint4 *>(gq_smem + L.xs_off);
    float *xsum = reinterpret_cast<float *>(gq_smem + L.xsum_off);
    for (int wi = warp; wi < cta_chunks * MT; wi += GQ_WARPS) {
        const int cc = wi / MT, m = wi - cc * MT;
        const uint8_t *src = xr + (m * 8 + g) * L.xr_stride + cc * 128 + t * 32;
        const uint4 r0 = *reinterpret_cast<const uint4 *>(src), r1 = *reinterpret_cast<const uint4 *>(src + 16);
        const uint4 f0 = make_uint4(prmt(r0.x, r0.z, 0x5410), prmt(r0.x, r0.z, 0x7632), prmt(r0.y, r0.w, 0x5410),
                                    prmt(r0.y, r0.w, 0x7632));
        const uint4 f1 = make_uint4(prmt(r1.x, r1.z, 0x5410), prmt(r1.x, r1.z, 0x7632), prmt(r1.y, r1.w, 0x5410),
                                    prmt(r1.y, r1.w, 0x7632));
        xs[((cc * MT + m) * 2) * 32 + lane] = f0;
        xs[((cc * MT + m) * 2 + 1) * 32 + lane] = f1;
        float X[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        mma_16816(X, ONES, ONES, ONES, ONES, f0.x, f0.y);
        mma_16816(X, ONES, ONES, ONES, ONES, f0.z, f0.w);
        mma_16816(X, ONES, ONES, ONES, ONES, f1.x, f1.y);
        mma_16816(X, ONES, ONES, ONES, ONES, f1.z, f1.w);
        if (g == 0) *reinterpret_cast<float2 *>(xsum + cc * 16 + m * 8 + 2 * t) = make_float2(X[0], X[1]);
    }
    __syncthreads();

    // Decode, multiply, apply each chunk's affine map.
    float acc[MT][4];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[m][i] = 0.0f;
#pragma unroll
    for (int j = 0; j < GQ_MAXC; ++j) {
        if (j < nch) {
            const int cc = cb + j - cta_lo;
            float P[MT][4];
#pragma unroll
            for (int m = 0; m < MT; ++m)
#pragma unroll
                for (int i = 0; i < 4; ++i) P[m][i] = 0.0f;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t wg = h ? cg[j].y : cg[j].x, wh = h ? ch[j].y : ch[j].x;
                const uint32_t g0 = nib_pair(wg), g1 = nib_pair(wg >> 4), g2 = nib_pair(wg >> 8),
                               g3 = nib_pair(wg >> 12);
                const uint32_t h0 = nib_pair(wh), h1 = nib_pair(wh >> 4), h2 = nib_pair(wh >> 8),
                               h3 = nib_pair(wh >> 12);
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    const uint4 xb = xs[((cc * MT + m) * 2 + h) * 32 + lane];
                    mma_16816(P[m], g0, h0, g1, h1, xb.x, xb.y);
                    mma_16816(P[m], g2, h2, g3, h3, xb.z, xb.w);
                }
            }
            const __half2 szg = *reinterpret_cast<const __half2 *>(&sg[j]);
            const __half2 szh = *reinterpret_cast<const __half2 *>(&sh[j]);
            const float s_g = __low2float(szg), zz_g = 128.0f + __high2float(szg);
            const float s_h = __low2float(szh), zz_h = 128.0f + __high2float(szh);
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                const float2 X = *reinterpret_cast<const float2 *>(xsum + cc * 16 + m * 8 + 2 * t);
                acc[m][0] = fmaf(s_g, fmaf(-zz_g, X.x, P[m][0]), acc[m][0]);
                acc[m][1] = fmaf(s_g, fmaf(-zz_g, X.y, P[m][1]), acc[m][1]);
                acc[m][2] = fmaf(s_h, fmaf(-zz_h, X.x, P[m][2]), acc[m][2]);
                acc[m][3] = fmaf(s_h, fmaf(-zz_h, X.y, P[m][3]), acc[m][3]);
            }
        }
    }

    // Partials of the CTA's warps: red[warp][row 16][token 16].
    float *red = reinterpret_cast<float *>(gq_smem + L.red_off);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        float *rw = red + warp * 256;
        *reinterpret_cast<float2 *>(rw + g * 16 + m * 8 + 2 * t) = make_float2(acc[m][0], acc[m][1]);
        *reinterpret_cast<float2 *>(rw + (g + 8) * 16 + m * 8 + 2 * t) = make_float2(acc[m][2], acc[m][3]);
    }
    __syncthreads();

    // From here on a thread handles one row and four tokens (float4 along
    // the tokens); consecutive threads take consecutive rows.
    const int M4 = (a.M + 3) / 4;
    auto cta_sum4 = [&](int rr, int q4) {  // CTA partial of group row rr, k-slices in order
        const int ti = rr >> 4, r = rr & 15;
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (int q = 0; q < ks; ++q) {
            const float4 u = *reinterpret_cast<const float4 *>(red + (q * rt + ti) * 256 + r * 16 + q4 * 4);
            v.x += u.x; v.y += u.y; v.z += u.z; v.w += u.w;
        }
        return v;
    };
    auto epilogue4 = [&](int lr, int q4, float4 v4) {  // lr: row among the ones this CTA finalises
        const int n = group_row0 + my_lo + lr;
        if (n >= a.N) return;
        const float vals[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int tok = q4 * 4 + i;
            if (tok >= a.M) break;
            float v = vals[i] + ep[lr];
            if (a.act == 1) v = gelu2(make_float2(v, v)).x;
            const int64_t yi = (a.y_row + tok) * (int64_t)a.N + n;
            if (a.gate) v = ld_elem_q(a.y, a.y_f32, yi) + v * ep[R + lr];
            if (a.y_f32) reinterpret_cast<float *>(a.y)[yi] = v;
            else reinterpret_cast<__nv_bfloat16 *>(a.y)[yi] = __float2bfloat16_rn(v);
        }
    };

    if (cs == 1) {
        for (int e = threadIdx.x; e < R * M4; e += GQ_THREADS) {
            const int rr = e % R, q4 = e / R;
            epilogue4(rr, q4, cta_sum4(rr, q4));
        }
        return;
    }

    // Cluster: rank o finalises group rows [o * rows_per, (o + 1) * rows_per);
    // every rank writes its partial for them into o's recv[src = own rank].
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");  // every CTA of the cluster runs
    const uint32_t recv_local = smem_u32(gq_smem + L.recv_off);
    for (int e = threadIdx.x; e < R * M4; e += GQ_THREADS) {
        const int rr = e % R, q4 = e / R;
        const int o = rr / rp;
        const float4 v = cta_sum4(rr, q4);
        const uint32_t off = (uint32_t)((crank * rp + (rr - o * rp)) * 16 + q4 * 4) * 4;
        const uint32_t dst = mapa_shared(recv_local + off, (uint32_t)o);
        asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "f"(v.x), "f"(v.y), "f"(v.z),
                     "f"(v.w)
                     : "memory");
    }
    cluster_sync();
    const float *recv = reinterpret_cast<const float *>(gq_smem + L.recv_off);
    for (int e = threadIdx.x; e < my_rows * M4; e += GQ_THREADS) {
        const int lr = e % my_rows, q4 = e / my_rows;
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (int src = 0; src < cs; ++src) {
            const float4 u = *reinterpret_cast<const float4 *>(recv + (src * rp + lr) * 16 + q4 * 4);
            v.x += u.x; v.y += u.y; v.z += u.z; v.w += u.w;
        }
        epilogue4(lr, q4, v);
    }
}

struct GqPlan {
    int rt, ks, cs, groups, maxc, cta_chunks;
};

// Pick the CTA shape: every warp's k-range within GQ_MAXC chunks and the
// shared memory within the per-CTA limit; then the least work on the busiest
// SM (CTAs per SM x (chunks per warp + a CTA's fixed part)), with a penalty
// when two CTAs' shared memory does not fit one SM (the next kernel's CTAs
// then cannot start beside them); then fewer row groups (each row group reads
// the whole of x once), then smaller clusters.
constexpr int GQ_SMEM_MAX = 227 * 1024;
constexpr int GQ_SMEM_HALF = 113 * 1024;
constexpr int GQ_CTA_CHUNKS = 4;

bool gq_plan(int N, int K, int num_sms, GqPlan &best) {
    const int T = (N + 15) / 16, C = K / 64;
    bool found = false;
    long long best_cost = 0;
    for (int rt = GQ_WARPS; rt >= 1; rt >>= 1) {
        const int ks = GQ_WARPS / rt;
        for (int cs = 1; cs <= GQ_MAXCS; ++cs) {
            const int S = ks * cs;
            if (S > C) break;
            const int maxc = (C + S - 1) / S;
            if (maxc > GQ_MAXC) continue;
            const int groups = (T + rt - 1) / rt;
            if (groups > 65535) continue;
            int cta_chunks = 0;
            for (int r = 0; r < cs; ++r) {
                const int c = slice_begin((r + 1) * ks, S, C) - slice_begin(r * ks, S, C);
                cta_chunks = c > cta_chunks ? c : cta_chunks;
            }
            const int bytes = gq_layout(2, cta_chunks, rt, cs).bytes;
            if (bytes > GQ_SMEM_MAX) continue;
            const long long ctas = (long long)groups * cs;
            const long long waves = (ctas + num_sms - 1) / num_sms;
            // a CTA's fixed part (x staging, reductions) ~ GQ_CTA_CHUNKS chunks
            const long long cost = ((waves * (maxc + GQ_CTA_CHUNKS) * (bytes <= GQ_SMEM_HALF ? 2 : 3)) << 40) +
                                   ((long long)groups << 8) + cs;
            if (!found || cost < best_cost) {
                best = GqPlan{rt, ks, cs, groups, maxc, cta_chunks};
                best_cost = cost;
                found = true;
            }
        }
    }
    return found;
}

std::atomic<int> g_gq_smem_optin[2][LX2V_MAX_DEVICES];

template <int MT>
cudaError_t gemv_q4_launch_t(const LinearArgs &a, const GqPlan &p, cudaStream_t st) {
    const GqLayout L = gq_layout(MT, p.cta_chunks, p.rt, p.cs);
    auto kern = gemv_q4_kernel<MT>;
    std::atomic<int> *slot = device_slot(g_gq_smem_optin[MT - 1]);
    if (!slot || slot->load() == 0) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, GQ_SMEM_MAX);
        if (e != cudaSuccess) return e;
        if (slot) slot->store(1);
    }
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof cfg);
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = p.cs;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.gridDim = dim3(p.cs, p.groups);
    cfg.blockDim = dim3(GQ_THREADS);
    cfg.dynamicSmemBytes = L.bytes;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kern, a, p.rt, p.ks, p.cs, p.cta_chunks);
}

}  // namespace

bool gemv_q4_supported(const LinearArgs &a, int num_sms) {
    if (a.fmt != FMT_Q4 || a.M < 1 || a.M > 16 || a.N < 1 || a.K < 64) return false;
    if (a.K % 64 != 0 || a.group % 64 != 0 || a.K % a.group != 0) return false;
    GqPlan p;
    return gq_plan(a.N, a.K, num_sms, p);
}

cudaError_t gemv_q4_launch(const LinearArgs &a, int num_sms, cudaStream_t st) {
    GqPlan p;
    if (!gq_plan(a.N, a.K, num_sms, p)) return cudaErrorInvalidValue;
    return a.M > 8 ? gemv_q4_launch_t<2>(a, p, st) : gemv_q4_launch_t<1>(a, p, st);
}

}  // namespace lx2v
