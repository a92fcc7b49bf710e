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
//               goes back through shared memory;
//   B operand = BT token rows of x (bf16, K-major), TMA-loaded into shared
//               memory with the 128-byte swizzle;
//   D         = 128 lanes (features) x BT columns (tokens) of f32 in TMEM.
// Each decoded weight value feeds BT tokens of MMA work.
//
// Per pipeline stage (one 64-wide k-block) TMA brings the x tile and the raw
// code tile of the 128 weight rows (64-, 32- or 128-byte swizzle so that the
// dequant threads' row reads are bank-conflict free).
//
// Warp roles (16 warps, one persistent CTA per SM):
//   warp 0      TMA producer (x tile + code tile per stage)
//   warp 1      TMEM allocator and MMA issuer (one thread)
//   warps 4-7   epilogue: TMEM -> registers -> bias/GELU/gate -> smem staging
//               -> TMA store (or TMA reduce-add for the gated residual)
//   warps 8-15  dequant: two warpgroups, each owns 32 of the 64 columns of a
//               k-block; thread = one weight row (TMEM lane)
// ACC accumulators (1 or 2) let the epilogue of tile j overlap the mainloop
// of tile j+1. Every mbarrier wait is bounded (ptx.cuh); on expiry the kernel
// records an error word, drains its own in-flight copies and MMAs, frees
// TMEM and returns.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <cstring>
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

// Bytes of one stage's code tile (128 weight rows x 64 k).
template <int FMT>
struct WTile {
    static constexpr int ROW_BYTES = FMT == FMT_Q4 ? 32 : FMT == FMT_BF16 ? 128 : 64;
    static constexpr int BYTES = 128 * ROW_BYTES;
};

template <int FMT, int BT, int ACC>
struct Cfg {
    static constexpr int A_COL0 = ACC * BT;  // first TMEM column of the A stages
    static_assert(A_COL0 + STAGES * (BK / 2) <= TMEM_COLS, "TMEM budget");
    static constexpr int X_STAGE_BYTES = BT * BK * 2;
    static constexpr int W_STAGE_BYTES = WTile<FMT>::BYTES;
    static constexpr int STAGE_TX = X_STAGE_BYTES + W_STAGE_BYTES;
    static constexpr int STG_BYTES = STG_ROWS * STG_COLS * 4;
    static constexpr int OFF_W = STAGES * X_STAGE_BYTES;
    static constexpr int OFF_STG = OFF_W + STAGES * W_STAGE_BYTES;
    static constexpr int OFF_BAR = OFF_STG + 2 * STG_BYTES;
    static constexpr int NUM_BARS = 3 * STAGES + 2 * ACC + 1;
    static constexpr int SMEM_BYTES = 1024 + OFF_BAR + NUM_BARS * 8 + 16;
    static_assert(X_STAGE_BYTES % 1024 == 0 && W_STAGE_BYTES % 1024 == 0, "swizzle atoms");
};

struct SmemCtl {
    uint32_t tmem_base;
    int epi_ok;
};

__device__ __forceinline__ float tanh_approx(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// GELU-tanh (crates/lightx2v-cpu/src/lib.rs:151-153) on a pair:
// 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))).
__device__ __forceinline__ float2 gelu2(float2 x) {
    const float2 c1 = make_float2(0.044715f, 0.044715f);
    const float2 one = make_float2(1.0f, 1.0f);
    const float2 k0 = make_float2(0.7978845608028654f, 0.7978845608028654f);
    const float2 half = make_float2(0.5f, 0.5f);
    const float2 x2 = __fmul2_rn(x, x);
    const float2 inner = __fmul2_rn(__fmul2_rn(x, k0), __ffma2_rn(x2, c1, one));
    const float2 t = make_float2(tanh_approx(inner.x), tanh_approx(inner.y));
    const float2 hx = __fmul2_rn(x, half);
    return __ffma2_rn(hx, t, hx);
}

__device__ __forceinline__ uint4 lds128(const uint8_t *p) {
    return *reinterpret_cast<const uint4 *>(p);
}

// Dequant warps: thread = one weight row (TMEM lane) of the 128-row tile;
// warpgroup `half` owns columns [32*half, 32*half + 32) of each k-block.
template <int FMT, int BT, int ACC>
__device__ __forceinline__ void dequant_role(const GemmParams &p, uint8_t *smem, uint32_t tmem,
                                             uint64_t *x_full, uint64_t *a_full, int warp, int lane,
                                             int n_mt, int KB, int total) {
    using C = Cfg<FMT, BT, ACC>;
    const int q = warp & 3;
    const int half = (warp - 8) >> 2;
    const int r = q * 32 + lane;  // row within the 128-row tile
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    const int ku = fp8_flag_cols(p.K);

    // Per-item side data (scales, flag), loaded one item ahead.
    auto side = [&](int it, float &s0, float &s1, float &z0, float &z1, bool &slow) {
        s0 = s1 = z0 = z1 = 0.0f;
        slow = false;
        if (it >= total) return;
        const int j = it / KB, kb = it - j * KB;
        const int tile = (int)blockIdx.x + j * (int)gridDim.x;
        const int n = (tile / n_mt) * 128 + r;
        const int kbase = kb * BK + half * 32;
        if (n >= p.N || kbase >= p.K) return;
        const int k1 = kbase + 16 < p.K ? kbase + 16 : kbase;
        const int64_t g0 = kbase / p.group, g1 = k1 / p.group;
        if (FMT == FMT_Q8 || FMT == FMT_FP8) {
            s0 = __ldg(p.scales_t + g0 * p.N + n);
            s1 = __ldg(p.scales_t + g1 * p.N + n);
            if (FMT == FMT_FP8) slow = __ldg(p.flags + (int64_t)n * ku + kbase / 32) != 0;
        } else if (FMT == FMT_Q4) {
            q4_scale_zero(__ldg(p.sz_t + g0 * p.N + n), s0, z0);
            q4_scale_zero(__ldg(p.sz_t + g1 * p.N + n), s1, z1);
        }
    };

    float s0, s1, z0, z1;
    bool slow;
    side(0, s0, s1, z0, z1, slow);
    for (int it = 0; it < total; ++it) {
        const int s = it % STAGES, rnd = it / STAGES;
        float ns0, ns1, nz0, nz1;
        bool nslow;
        side(it + 1, ns0, ns1, nz0, nz1, nslow);

        int ok = 1;
        if (lane == 0) ok = mbar_wait_bounded(&x_full[s], rnd & 1, p.err, p.wait_limit_ns) ? 1 : 0;
        ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
        if (!ok) return;

        const uint8_t *wt = smem + C::OFF_W + s * C::W_STAGE_BYTES + r * WTile<FMT>::ROW_BYTES;
        uint32_t packed[16];
        if (FMT == FMT_Q4) {
            // 32-byte rows, 32B swizzle: chunk ^= (row >> 2) & 1
            const uint4 raw = lds128(wt + ((half ^ ((r >> 2) & 1)) << 4));
            uint32_t o0[8], o1[8];
            unit_to_bf16<FMT_Q4>(make_uint4(raw.x, raw.y, 0, 0), raw, s0, z0, false, o0);
            unit_to_bf16<FMT_Q4>(make_uint4(raw.z, raw.w, 0, 0), raw, s1, z1, false, o1);
#pragma unroll
            for (int i = 0; i < 8; ++i) { packed[i] = o0[i]; packed[8 + i] = o1[i]; }
        } else if (FMT == FMT_BF16) {
            // 128-byte rows, 128B swizzle: chunk ^= row & 7
            const int c0 = half * 4;
            uint4 v[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] = lds128(wt + (((c0 + i) ^ (r & 7)) << 4));
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                packed[4 * i] = v[i].x; packed[4 * i + 1] = v[i].y;
                packed[4 * i + 2] = v[i].z; packed[4 * i + 3] = v[i].w;
            }
        } else {
            // 64-byte rows, 64B swizzle: chunk ^= (row >> 1) & 3
            const int sw = (r >> 1) & 3;
            const uint4 a = lds128(wt + (((half * 2) ^ sw) << 4));
            const uint4 b = lds128(wt + (((half * 2 + 1) ^ sw) << 4));
            uint32_t o0[8], o1[8];
            unit_to_bf16<FMT>(a, a, s0, 0.0f, slow, o0);
            unit_to_bf16<FMT>(b, b, s1, 0.0f, slow, o1);
#pragma unroll
            for (int i = 0; i < 8; ++i) { packed[i] = o0[i]; packed[8 + i] = o1[i]; }
        }
        tmem_st_32x32b_x16(tmem + lane_addr + (uint32_t)(C::A_COL0 + s * (BK / 2) + half * 16), packed);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[s]);
        s0 = ns0; s1 = ns1; z0 = nz0; z1 = nz1; slow = nslow;
    }
}

template <int FMT, int BT, int ACC>
__global__ void __launch_bounds__(NUM_THREADS, 1) gemm_dq_kernel(const __grid_constant__ GemmParams p) {
    using C = Cfg<FMT, BT, ACC>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::OFF_BAR);
    uint64_t *x_full = bars;                        // [STAGES] TMA tx (x + codes)
    uint64_t *a_full = bars + STAGES;               // [STAGES] 8 dequant warps
    uint64_t *st_empty = bars + 2 * STAGES;         // [STAGES] MMA commit
    uint64_t *acc_full = bars + 3 * STAGES;         // [ACC] MMA commit
    uint64_t *acc_empty = acc_full + ACC;           // [ACC] 4 epilogue warps
    uint64_t *drain = acc_empty + ACC;              // [1] final MMA drain
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
        for (int b = 0; b < ACC; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 4);
        }
        mbar_init(drain, 1);
        fence_mbar_init();
        tma_prefetch_desc(&p.tmap_x);
        tma_prefetch_desc(&p.tmap_w);
        tma_prefetch_desc(&p.tmap_y);
    }
    if (warp == 1) tmem_alloc(&ctl->tmem_base, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;

    if (warp == 0) {
        // ---------------- TMA producer: x tile + code tile ----------------
        if (lane == 0) {
            int last_round[STAGES];
            for (int s = 0; s < STAGES; ++s) last_round[s] = -1;
            const int wk_div = FMT == FMT_Q4 ? 2 : 1;  // the Q4 code map counts bytes (2 values)
            for (int it = 0; it < total; ++it) {
                const int j = it / KB, kb = it - j * KB;
                const int tile = (int)blockIdx.x + j * (int)gridDim.x;
                const int mt = tile % n_mt, ft = tile / n_mt;
                const int s = it % STAGES, r = it / STAGES;
                if (!mbar_wait_bounded(&st_empty[s], (r & 1) ^ 1, err, lim)) break;
                mbar_arrive_expect_tx(&x_full[s], C::STAGE_TX);
                tma_load_2d(smem + s * C::X_STAGE_BYTES, &p.tmap_x, &x_full[s], kb * BK, p.x_row + mt * BT);
                tma_load_2d(smem + C::OFF_W + s * C::W_STAGE_BYTES, &p.tmap_w, &x_full[s],
                            kb * BK / wk_div, ft * 128);
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
                const int b = j % ACC, rb = j / ACC;
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
            const int b = j % ACC, rb = j / ACC;
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
            const float2 bias2 = make_float2(bias_f, bias_f), gate2 = make_float2(gate_f, gate_f);
            const int m0 = mt * BT;
            const int nch = min(BT / 32, (p.M - m0 + 31) / 32);
            for (int c = 0; c < nch; ++c) {
                uint32_t acc[32];
                tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * BT + c * 32), acc);
                tmem_wait_ld();
                if (c == nch - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&acc_empty[b]);
                }
                float2 v[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    float2 t = __fadd2_rn(make_float2(__uint_as_float(acc[2 * i]), __uint_as_float(acc[2 * i + 1])), bias2);
                    if (p.act == 1) t = gelu2(t);
                    v[i] = p.gate ? __fmul2_rn(t, gate2) : t;
                }
                const int pb = chunk_ctr & 1;
                ++chunk_ctr;
                uint8_t *stg = smem + C::OFF_STG + pb * C::STG_BYTES;
                if (leader) bulk_wait_read<1>();
                named_bar_sync(1, EPI_THREADS);
                if (out_f32) {
                    float *s32 = reinterpret_cast<float *>(stg) + q * 32 + lane;
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        s32[(2 * i) * STG_COLS] = v[i].x;
                        s32[(2 * i + 1) * STG_COLS] = v[i].y;
                    }
                } else {
                    unsigned short *s16 = reinterpret_cast<unsigned short *>(stg) + q * 32 + lane;
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const uint32_t pk = pack_bf16x2(v[i]);
                        s16[(2 * i) * STG_COLS] = (unsigned short)(pk & 0xFFFFu);
                        s16[(2 * i + 1) * STG_COLS] = (unsigned short)(pk >> 16);
                    }
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
        dequant_role<FMT, BT, ACC>(p, smem, tmem, x_full, a_full, warp, lane, n_mt, KB, total);
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

// ---- host launcher --------------------------------------------------------
template <int FMT, int BT, int ACC>
static cudaError_t launch_t(const GemmParams &p, int num_sms, cudaStream_t st) {
    using C = Cfg<FMT, BT, ACC>;
    static bool attr_set = false;
    // Keep the footprint large enough that only one CTA fits per SM: each
    // CTA allocates all 512 TMEM columns.
    const int smem = C::SMEM_BYTES > 120 * 1024 ? C::SMEM_BYTES : 120 * 1024;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(gemm_dq_kernel<FMT, BT, ACC>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    const int n_tiles = ((p.M + BT - 1) / BT) * ((p.N + 127) / 128);
    const int grid = n_tiles < num_sms ? n_tiles : num_sms;
    gemm_dq_kernel<FMT, BT, ACC><<<grid, NUM_THREADS, smem, st>>>(p);
    return cudaGetLastError();
}

template <int FMT>
static cudaError_t launch_fmt(int bt, const GemmParams &p, int num_sms, cudaStream_t st) {
    switch (bt) {
        case 128: return launch_t<FMT, 128, 2>(p, num_sms, st);
        case 192: return launch_t<FMT, 192, 2>(p, num_sms, st);
        case 256: return launch_t<FMT, 256, 1>(p, num_sms, st);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t gemm_dq_launch(int fmt, int bt, const GemmParams &p, int num_sms, cudaStream_t st) {
    switch (fmt) {
        case FMT_Q8: return launch_fmt<FMT_Q8>(bt, p, num_sms, st);
        case FMT_Q4: return launch_fmt<FMT_Q4>(bt, p, num_sms, st);
        case FMT_FP8: return launch_fmt<FMT_FP8>(bt, p, num_sms, st);
        default: return launch_fmt<FMT_BF16>(bt, p, num_sms, st);
    }
}

int gemm_dq_token_tile(int M, int N, int num_sms) {
    // Pick the token tile that minimises (waves x tile width): the kernel is
    // paced per tile by the MMA work, which is proportional to the width.
    const int cands[3] = {256, 192, 128};
    int best = 128;
    double best_cost = 1e30;
    const int n_ft = (N + 127) / 128;
    for (int bt : cands) {
        const int tiles = ((M + bt - 1) / bt) * n_ft;
        const int waves = (tiles + num_sms - 1) / num_sms;
        // wider tiles amortise the weight decode over more tokens
        const double cost = (double)waves * bt * (1.0 + 32.0 / bt);
        if (cost < best_cost - 1e-9) { best_cost = cost; best = bt; }
    }
    return best;
}

}  // namespace lx2v
