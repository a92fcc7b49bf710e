// gemm_sm100.cu — the quantized linear on tcgen05 tensor cores (sm_100a).
//
// Computes Backend::linear (crates/lightx2v-core/src/backend.rs:199-212)
//   y[y_row + m, n] = act(sum_k x[x_row + m, k] * W[n, k] + bias[n])
// for W in any of the reference's formats (Q8, Q4, FP8 e4m3, native), and
// the fused linear + gate_residual (backend.rs:244-253) where the epilogue
// reduce-adds gate[n] * act(...) into h.
//
// Orientation. The tensor core computes D^T = W_tile * X_tile^T:
//   A operand = 128 weight rows (features), taken from TENSOR MEMORY. The
//               dequant warps decode packed codes in registers and tcgen05.st
//               the bf16 values straight into TMEM, so a decoded weight never
//               touches shared memory;
//   B operand = BT token rows of x (bf16, K-major), TMA-loaded into shared
//               memory with the 128-byte swizzle;
//   D         = 128 lanes (features) x BT columns (tokens) of f32 in TMEM.
// Each decoded weight value feeds BT tokens, so the per-value decode cost is
// spread over BT MMA columns.
//
// Warp roles (16 warps, one persistent CTA per SM):
//   warp 0      TMA producer of x tiles
//   warp 1      TMEM allocator and MMA issuer (one thread)
//   warps 4-7   epilogue: TMEM -> registers -> bias/GELU/gate -> smem staging
//               -> TMA store (or TMA reduce-add for the gated residual)
//   warps 8-15  dequant: two warpgroups, each owns half of a 64-wide k-block;
//               thread = one weight row (TMEM lane)
// Pipelines: STAGES-deep ring of (x smem tile, A TMEM tile), and ACC_BUFS
// accumulators so the epilogue of tile j overlaps the mainloop of tile j+1.
// Every mbarrier wait is bounded (ptx.cuh); on expiry the kernel records an
// error word, drains its own in-flight copies and MMAs, frees TMEM, returns.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>
#include "dequant.cuh"
#include "gemm.h"
#include "ptx.cuh"

namespace lx2v {

constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int NUM_THREADS = 512;
constexpr int EPI_THREADS = 128;
constexpr int STG_ROWS = 32;      // tokens per epilogue staging chunk
constexpr int STG_COLS = 128;     // features per staging chunk
constexpr int TMEM_COLS = 512;

template <int BT>
struct Cfg {
    static constexpr int ACC_BUFS = (BT <= 192) ? 2 : 1;
    static constexpr int A_COL0 = ACC_BUFS * BT;  // first TMEM column of the A stages
    static_assert(A_COL0 + STAGES * (BK / 2) <= TMEM_COLS, "TMEM budget");
    static constexpr int X_STAGE_BYTES = BT * BK * 2;
    static constexpr int STG_BYTES = STG_ROWS * STG_COLS * 4;
    static constexpr int OFF_STG = STAGES * X_STAGE_BYTES;
    static constexpr int OFF_BAR = OFF_STG + 2 * STG_BYTES;
    static constexpr int NUM_BARS = 3 * STAGES + 2 * ACC_BUFS + 1;
    static constexpr int SMEM_BYTES = 1024 + OFF_BAR + NUM_BARS * 8 + 16;
};

struct SmemCtl {
    uint32_t tmem_base;
    int epi_ok;
};

__device__ __forceinline__ float gelu_tanh_dev(float x) {
    // 0.5 x (1 + tanh(u)) == x * sigmoid(2u), u = sqrt(2/pi) (x + 0.044715 x^3)
    // (crates/lightx2v-cpu/src/lib.rs:151-153); written with exp so that it is
    // one MUFU exp and one reciprocal.
    const float u = 0.7978845608028654f * (x + 0.044715f * x * x * x);
    return __fdividef(x, 1.0f + __expf(-2.0f * u));
}

// Raw (undecoded) data of one work item for one dequant thread: 32 values
// of one weight row (two 16-value units) plus their scales.
template <int FMT>
struct Raw {
    uint4 a, b, c, d;   // Q8/FP8 use a,b; Q4 uses a.x..a.w; BF16 uses a..d
    uint32_t s0, s1;    // Q8/FP8 scale bits or Q4 half2 (scale, zero), per unit
};

template <int FMT>
__device__ __forceinline__ void raw_load(const GemmParams &p, int n, int kbase, Raw<FMT> &r) {
    if (n >= p.N || kbase >= p.K) {
        r.a = r.b = r.c = r.d = make_uint4(0, 0, 0, 0);
        r.s0 = r.s1 = 0;
        return;
    }
    const int64_t base = (int64_t)n * p.K + kbase;
    const bool u1 = kbase + 16 < p.K;   // second unit inside the row
    const int g0 = kbase / p.group, g1 = (kbase + 16) / p.group;
    if (FMT == FMT_Q8 || FMT == FMT_FP8) {
        const uint4 *src = reinterpret_cast<const uint4 *>(p.codes + base);
        r.a = __ldg(src);
        r.b = u1 ? __ldg(src + 1) : make_uint4(0, 0, 0, 0);
        r.s0 = __float_as_uint(__ldg(p.scales_t + (int64_t)g0 * p.N + n));
        r.s1 = u1 ? __float_as_uint(__ldg(p.scales_t + (int64_t)g1 * p.N + n)) : 0u;
    } else if (FMT == FMT_Q4) {
        const uint2 *src = reinterpret_cast<const uint2 *>(p.codes + base / 2);
        const uint2 lo = __ldg(src);
        const uint2 hi = u1 ? __ldg(src + 1) : make_uint2(0, 0);
        r.a = make_uint4(lo.x, lo.y, hi.x, hi.y);
        r.s0 = __ldg(p.sz_t + (int64_t)g0 * p.N + n);
        r.s1 = u1 ? __ldg(p.sz_t + (int64_t)g1 * p.N + n) : 0u;
    } else {
        const uint4 *src = reinterpret_cast<const uint4 *>(reinterpret_cast<const __nv_bfloat16 *>(p.codes) + base);
        r.a = __ldg(src);
        r.b = __ldg(src + 1);
        r.c = u1 ? __ldg(src + 2) : make_uint4(0, 0, 0, 0);
        r.d = u1 ? __ldg(src + 3) : make_uint4(0, 0, 0, 0);
    }
}

// Decode one item into 16 bf16x2 words (column pairs k, k+1 -> lo, hi).
template <int FMT>
__device__ __forceinline__ void raw_decode(const GemmParams &p, const Raw<FMT> &r, uint32_t (&packed)[16]) {
    if (FMT == FMT_BF16) {
        const uint4 v[4] = {r.a, r.b, r.c, r.d};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            packed[4 * i + 0] = v[i].x; packed[4 * i + 1] = v[i].y;
            packed[4 * i + 2] = v[i].z; packed[4 * i + 3] = v[i].w;
        }
        return;
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        float vals[16];
        const uint32_t sb = u ? r.s1 : r.s0;
        if (FMT == FMT_Q8) {
            dq_q8_unit(u ? r.b : r.a, __uint_as_float(sb), vals);
        } else if (FMT == FMT_FP8) {
            dq_fp8_unit(u ? r.b : r.a, __uint_as_float(sb), p.fp8_fast != 0, vals);
        } else {
            float s, z;
            q4_scale_zero(sb, s, z);
            dq_q4_unit(u ? make_uint2(r.a.z, r.a.w) : make_uint2(r.a.x, r.a.y), s, z, vals);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) packed[u * 8 + i] = pack_bf16x2(vals[2 * i], vals[2 * i + 1]);
    }
}

// Dequant warps: thread = one weight row (TMEM lane) of the 128-row tile,
// warpgroup `half` owns columns [32*half, 32*half+32) of each 64-wide
// k-block. Raw codes are prefetched PF items ahead in registers.
template <int FMT, int BT>
__device__ __forceinline__ void dequant_role(const GemmParams &p, uint32_t tmem, uint64_t *st_empty,
                                             uint64_t *a_full, int warp, int lane, int n_mt, int KB,
                                             int total) {
    constexpr int PF = 4;
    const int q = warp & 3;
    const int half = (warp - 8) >> 2;
    const int row_in_tile = q * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    auto item_coords = [&](int it, int &n, int &kbase) {
        const int j = it / KB, kb = it - j * KB;
        const int tile = (int)blockIdx.x + j * (int)gridDim.x;
        n = (tile / n_mt) * 128 + row_in_tile;
        kbase = kb * BK + half * 32;
    };
    Raw<FMT> ring[PF];
#pragma unroll
    for (int d = 0; d < PF; ++d) {
        int n = p.N, kbase = 0;
        if (d < total) item_coords(d, n, kbase);
        raw_load<FMT>(p, n, kbase, ring[d]);
    }
    for (int it0 = 0; it0 < total; it0 += PF) {
#pragma unroll
        for (int d = 0; d < PF; ++d) {
            const int it = it0 + d;
            if (it >= total) return;
            uint32_t packed[16];
            raw_decode<FMT>(p, ring[d], packed);
            {
                int n = p.N, kbase = 0;
                if (it + PF < total) item_coords(it + PF, n, kbase);
                raw_load<FMT>(p, n, kbase, ring[d]);
            }
            const int s = it % STAGES, r = it / STAGES;
            int ok = 1;
            if (lane == 0) ok = mbar_wait_bounded(&st_empty[s], (r & 1) ^ 1, p.err, p.wait_limit_ns) ? 1 : 0;
            ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
            if (!ok) return;
            tc_fence_after();
            tmem_st_32x32b_x16(tmem + lane_addr + (uint32_t)(Cfg<BT>::A_COL0 + s * (BK / 2) + half * 16), packed);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&a_full[s]);
        }
    }
}

template <int FMT, int BT>
__global__ void __launch_bounds__(NUM_THREADS, 1) gemm_dq_kernel(const __grid_constant__ GemmParams p) {
    using C = Cfg<BT>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::OFF_BAR);
    uint64_t *x_full = bars;                        // [STAGES] TMA tx
    uint64_t *a_full = bars + STAGES;               // [STAGES] 8 dequant warps
    uint64_t *st_empty = bars + 2 * STAGES;         // [STAGES] MMA commit
    uint64_t *acc_full = bars + 3 * STAGES;         // [ACC_BUFS] MMA commit
    uint64_t *acc_empty = acc_full + C::ACC_BUFS;   // [ACC_BUFS] 4 epilogue warps
    uint64_t *drain = acc_empty + C::ACC_BUFS;      // [1] final MMA drain
    SmemCtl *ctl = reinterpret_cast<SmemCtl *>(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_mt = (p.M + BT - 1) / BT;
    const int n_ft = (p.N + 127) / 128;
    const int n_tiles = n_mt * n_ft;
    const int KB = (p.K + BK - 1) / BK;
    const int my_tiles = (int)blockIdx.x < n_tiles ? (n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int total = my_tiles * KB;
    int *err = p.err;
    const uint64_t lim = p.wait_limit_ns;
    // Drains after an abort wait for copies / MMAs this CTA issued itself;
    // those finish in microseconds, so they get at least half a second even
    // when the pipeline limit is set very short.
    const uint64_t drain_lim = lim > 500000000ull ? lim : 500000000ull;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&x_full[s], 1);
            mbar_init(&a_full[s], 8);
            mbar_init(&st_empty[s], 1);
        }
        for (int b = 0; b < C::ACC_BUFS; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 4);
        }
        mbar_init(drain, 1);
        fence_mbar_init();
        tma_prefetch_desc(&p.tmap_x);
        tma_prefetch_desc(&p.tmap_y);
    }
    if (warp == 1) tmem_alloc(&ctl->tmem_base, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;

    if (warp == 0) {
        // ---------------- TMA producer: x tiles ----------------
        if (lane == 0) {
            int last_round[STAGES];
            for (int s = 0; s < STAGES; ++s) last_round[s] = -1;
            for (int it = 0; it < total; ++it) {
                const int j = it / KB, kb = it - j * KB;
                const int tile = (int)blockIdx.x + j * (int)gridDim.x;
                const int mt = tile % n_mt;
                const int s = it % STAGES, r = it / STAGES;
                if (!mbar_wait_bounded(&st_empty[s], (r & 1) ^ 1, err, lim)) break;
                mbar_arrive_expect_tx(&x_full[s], C::X_STAGE_BYTES);
                tma_load_2d(smem + s * C::X_STAGE_BYTES, &p.tmap_x, &x_full[s], kb * BK,
                            p.x_row + mt * BT);
                last_round[s] = r;
            }
            // Drain: every issued load has landed before smem can be released.
            for (int s = 0; s < STAGES; ++s)
                if (last_round[s] >= 0) mbar_wait_bounded(&x_full[s], last_round[s] & 1, nullptr, drain_lim);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = idesc_bf16_f32(128, BT);
            bool ok = true;
            for (int j = 0; j < my_tiles && ok; ++j) {
                const int b = j % C::ACC_BUFS, rb = j / C::ACC_BUFS;
                if (!mbar_wait_bounded(&acc_empty[b], (rb & 1) ^ 1, err, lim)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem + (uint32_t)(b * BT);
                for (int kb = 0; kb < KB; ++kb) {
                    const int it = j * KB + kb;
                    const int s = it % STAGES, r = it / STAGES;
                    if (!mbar_wait_bounded(&x_full[s], r & 1, err, lim) ||
                        !mbar_wait_bounded(&a_full[s], r & 1, err, lim)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a_tmem = tmem + (uint32_t)(C::A_COL0 + s * (BK / 2));
                    const uint64_t b_desc = smem_desc_sw128(smem_u32(smem + s * C::X_STAGE_BYTES));
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk)
                        mma_ts_f16(d_tmem, a_tmem + kk * 8, b_desc + (uint64_t)(kk * 2), idesc,
                                   (kb | kk) != 0);
                    mma_commit(&st_empty[s]);
                }
                if (!ok) break;
                mma_commit(&acc_full[b]);
            }
            // Drain: all MMAs issued by this thread complete before TMEM is freed.
            mma_commit(drain);
            mbar_wait_bounded(drain, 0, nullptr, drain_lim);
        }
        __syncwarp();
    } else if (warp >= 4 && warp < 8) {
        // ---------------- epilogue ----------------
        const int q = warp - 4;
        const bool leader = threadIdx.x == 128;
        int chunk_ctr = 0;
        const bool out_f32 = p.out_f32 != 0;
        for (int j = 0; j < my_tiles; ++j) {
            const int tile = (int)blockIdx.x + j * (int)gridDim.x;
            const int mt = tile % n_mt, ft = tile / n_mt;
            const int b = j % C::ACC_BUFS, rb = j / C::ACC_BUFS;
            if (leader) ctl->epi_ok = mbar_wait_bounded(&acc_full[b], rb & 1, err, lim) ? 1 : 0;
            named_bar_sync(1, EPI_THREADS);
            if (!ctl->epi_ok) break;
            tc_fence_after();
            const int f = ft * 128 + q * 32 + lane;
            float bias_f = 0.0f, gate_f = 1.0f;
            if (f < p.N) {
                if (p.bias) bias_f = p.bias_f32 ? reinterpret_cast<const float *>(p.bias)[f]
                                                : __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p.bias)[f]);
                if (p.gate) gate_f = p.gate_f32 ? reinterpret_cast<const float *>(p.gate)[f]
                                                : __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p.gate)[f]);
            }
            const int m0 = mt * BT;
            const int rows_left = p.M - m0;
            const int nch = min(BT / 32, (rows_left + 31) / 32);
            for (int c = 0; c < nch; ++c) {
                uint32_t acc[32];
                tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * BT + c * 32), acc);
                tmem_wait_ld();
                if (c == nch - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&acc_empty[b]);
                }
                float v[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    float t = __uint_as_float(acc[i]) + bias_f;
                    if (p.act == 1) t = gelu_tanh_dev(t);
                    v[i] = t * gate_f;
                }
                const int pb = chunk_ctr & 1;
                ++chunk_ctr;
                uint8_t *stg = smem + C::OFF_STG + pb * C::STG_BYTES;
                if (leader) bulk_wait_read<1>();
                named_bar_sync(1, EPI_THREADS);
                if (out_f32) {
                    float *s32 = reinterpret_cast<float *>(stg);
#pragma unroll
                    for (int i = 0; i < 32; ++i) s32[i * STG_COLS + q * 32 + lane] = v[i];
                } else {
                    __nv_bfloat16 *s16 = reinterpret_cast<__nv_bfloat16 *>(stg);
#pragma unroll
                    for (int i = 0; i < 32; ++i) s16[i * STG_COLS + q * 32 + lane] = __float2bfloat16_rn(v[i]);
                }
                fence_proxy_async_smem();
                named_bar_sync(1, EPI_THREADS);
                if (leader) {
                    const int c0 = ft * 128, c1 = p.y_row + m0 + c * 32;
                    if (p.reduce) tma_reduce_add_2d(&p.tmap_y, stg, c0, c1);
                    else tma_store_2d(&p.tmap_y, stg, c0, c1);
                    bulk_commit();
                }
            }
        }
        if (leader) bulk_wait<0>();
    } else if (warp >= 8) {
        // ---------------- dequant: codes -> bf16 -> TMEM (A operand) ----------------
        dequant_role<FMT, BT>(p, tmem, st_empty, a_full, warp, lane, n_mt, KB, total);
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

// ---- host launcher --------------------------------------------------------
template <int FMT, int BT>
static cudaError_t launch_t(const GemmParams &p, int num_sms, cudaStream_t st) {
    using C = Cfg<BT>;
    static bool attr_set = false;  // per process; harmless to repeat
    // Keep the footprint large enough that only one CTA fits per SM: each
    // CTA allocates all 512 TMEM columns.
    const int smem = C::SMEM_BYTES > 120 * 1024 ? C::SMEM_BYTES : 120 * 1024;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(gemm_dq_kernel<FMT, BT>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    const int n_tiles = ((p.M + BT - 1) / BT) * ((p.N + 127) / 128);
    const int grid = n_tiles < num_sms ? n_tiles : num_sms;
    gemm_dq_kernel<FMT, BT><<<grid, NUM_THREADS, smem, st>>>(p);
    return cudaGetLastError();
}

template <int BT>
static cudaError_t launch_bt(int fmt, const GemmParams &p, int num_sms, cudaStream_t st) {
    switch (fmt) {
        case FMT_Q8: return launch_t<FMT_Q8, BT>(p, num_sms, st);
        case FMT_Q4: return launch_t<FMT_Q4, BT>(p, num_sms, st);
        case FMT_FP8: return launch_t<FMT_FP8, BT>(p, num_sms, st);
        default: return launch_t<FMT_BF16, BT>(p, num_sms, st);
    }
}

cudaError_t gemm_dq_launch(int fmt, int bt, const GemmParams &p, int num_sms, cudaStream_t st) {
    switch (bt) {
        case 128: return launch_bt<128>(fmt, p, num_sms, st);
        case 192: return launch_bt<192>(fmt, p, num_sms, st);
        case 256: return launch_bt<256>(fmt, p, num_sms, st);
        default: return cudaErrorInvalidValue;
    }
}

int gemm_dq_token_tile(int M) {
    // A whole-M tile count that is no larger than needed; prefer the widest
    // token tile while it does not waste more than ~1/8 of a tile.
    if (M >= 256 * 8) return 256;
    if (M >= 192 * 4) return 192;
    return 128;
}

}  // namespace lx2v
