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
constexpr int NUM_THREADS = 512;
constexpr int EPI_THREADS = 128;
constexpr int STG_ROWS = 16;    // tokens per epilogue staging chunk (half a 32-column TMEM load)
constexpr int STG_COLS = 128;   // features per staging chunk
constexpr int TMEM_COLS = 512;

// Bytes of one stage's code tile (128 weight rows x 64 k) and of its side
// data: scales (Q8/FP8 f32, Q4 (scale, zero) words) for up to SGRP groups,
// and the FP8 block flags of the two 32-column halves.
template <int FMT>
struct WTile {
    static constexpr int ROW_BYTES = FMT == FMT_Q4 ? 32 : FMT == FMT_BF16 ? 128 : 64;
    static constexpr int BYTES = 128 * ROW_BYTES;
    static constexpr int SGRP = FMT == FMT_Q4 ? 4 : FMT == FMT_BF16 ? 0 : 1;
    static constexpr int S_BYTES = 128 * 4 * SGRP;
    static constexpr int F_BYTES = FMT == FMT_FP8 ? 2 * 128 : 0;
};

// SS = shared-memory stages (x tile + code tile), AS = TMEM stages of the
// decoded A operand, ACC = accumulators of BT columns each.
template <int FMT, int BT, int ACC, int SS, int AS>
struct Cfg {
    static constexpr int A_COL0 = ACC * BT;  // first TMEM column of the A stages
    static_assert(A_COL0 + AS * (BK / 2) <= TMEM_COLS, "TMEM budget");
    static constexpr int X_STAGE_BYTES = BT * BK * 2;
    static constexpr int W_STAGE_BYTES = WTile<FMT>::BYTES;
    static constexpr int S_STAGE_BYTES = WTile<FMT>::S_BYTES;
    static constexpr int F_STAGE_BYTES = WTile<FMT>::F_BYTES;
    static constexpr int STG_BYTES = STG_ROWS * STG_COLS * 4;
    static constexpr int OFF_W = SS * X_STAGE_BYTES;
    static constexpr int OFF_S = OFF_W + SS * W_STAGE_BYTES;
    static constexpr int OFF_F = OFF_S + SS * S_STAGE_BYTES;
    static constexpr int OFF_STG = (OFF_F + SS * F_STAGE_BYTES + 127) & ~127;
    static constexpr int OFF_BAR = OFF_STG + 2 * STG_BYTES;
    static constexpr int NUM_BARS = 2 * SS + 2 * AS + 2 * ACC + 1;
    static constexpr int SMEM_BYTES = 1024 + OFF_BAR + NUM_BARS * 8 + 16;
    static_assert(X_STAGE_BYTES % 1024 == 0 && W_STAGE_BYTES % 1024 == 0, "swizzle atoms");
    static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
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

// A ring position (stage, phase) advanced per item without divisions.
struct Ring {
    int s = 0, ph = 0;
    template <int N>
    __device__ __forceinline__ void next() {
        if (++s == N) { s = 0; ph ^= 1; }
    }
};

// Dequant warps: thread = one weight row (TMEM lane) of the 128-row tile;
// warpgroup `half` owns columns [32*half, 32*half + 32) of each k-block.
template <int FMT, int BT, int ACC, int SS, int AS>
__device__ __forceinline__ void dequant_role(const GemmParams &p, uint8_t *smem, uint32_t tmem,
                                             uint64_t *x_full, uint64_t *a_full, uint64_t *a_empty,
                                             int warp, int lane, int KB, int my_tiles) {
    using C = Cfg<FMT, BT, ACC, SS, AS>;
    const int q = warp & 3;
    const int half = (warp - 8) >> 2;
    const int r = q * 32 + lane;  // row within the 128-row tile
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    Ring xs, as;
    for (int j = 0; j < my_tiles; ++j) {
        for (int kb = 0; kb < KB; ++kb) {
            int ok = 1;
            if (lane == 0) ok = mbar_wait_bounded(&x_full[xs.s], xs.ph, p.err, p.wait_limit_ns) ? 1 : 0;
            ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
            if (!ok) return;

            const uint8_t *wt = smem + C::OFF_W + xs.s * C::W_STAGE_BYTES + r * WTile<FMT>::ROW_BYTES;
            // Side data of this row from the stage: scale word(s) of the
            // groups of the two 16-column units, and the FP8 block flag.
            float s0 = 0.0f, s1 = 0.0f, z0 = 0.0f, z1 = 0.0f;
            int mode = 0;
            if (FMT != FMT_BF16) {
                const uint32_t *sw = reinterpret_cast<const uint32_t *>(smem + C::OFF_S + xs.s * C::S_STAGE_BYTES);
                const int kbase = kb * BK + half * 32;
                const int gbase = (kb * BK) / p.group;
                const int gi0 = kbase / p.group - gbase, gi1 = (kbase + 16) / p.group - gbase;
                const int i0 = gi0 < WTile<FMT>::SGRP ? gi0 : 0, i1 = gi1 < WTile<FMT>::SGRP ? gi1 : 0;
                if (FMT == FMT_Q4) {
                    q4_scale_zero(sw[i0 * 128 + r], s0, z0);
                    q4_scale_zero(sw[i1 * 128 + r], s1, z1);
                } else {
                    s0 = __uint_as_float(sw[i0 * 128 + r]);
                    s1 = __uint_as_float(sw[i1 * 128 + r]);
                }
                if (FMT == FMT_FP8) mode = (smem + C::OFF_F + xs.s * C::F_STAGE_BYTES)[half * 128 + r];
            }
            uint32_t packed[16];
            if (FMT == FMT_Q4) {
                // 32-byte rows, 32B swizzle: chunk ^= (row >> 2) & 1
                const uint4 raw = lds128(wt + ((half ^ ((r >> 2) & 1)) << 4));
                uint32_t o0[8], o1[8];
                unit_to_bf16<FMT_Q4>(make_uint4(raw.x, raw.y, 0, 0), raw, s0, z0, 0, o0);
                unit_to_bf16<FMT_Q4>(make_uint4(raw.z, raw.w, 0, 0), raw, s1, z1, 0, o1);
#pragma unroll
                for (int i = 0; i < 8; ++i) { packed[i] = o0[i]; packed[8 + i] = o1[i]; }
            } else if (FMT == FMT_BF16) {
                // 128-byte rows, 128B swizzle: chunk ^= row & 7
                const int c0 = half * 4;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint4 v = lds128(wt + (((c0 + i) ^ (r & 7)) << 4));
                    packed[4 * i] = v.x; packed[4 * i + 1] = v.y;
                    packed[4 * i + 2] = v.z; packed[4 * i + 3] = v.w;
                }
            } else {
                // 64-byte rows, 64B swizzle: chunk ^= (row >> 1) & 3
                const int sw = (r >> 1) & 3;
                const uint4 a = lds128(wt + (((half * 2) ^ sw) << 4));
                const uint4 b = lds128(wt + (((half * 2 + 1) ^ sw) << 4));
                uint32_t o0[8], o1[8];
                unit_to_bf16<FMT>(a, a, s0, 0.0f, mode, o0);
                unit_to_bf16<FMT>(b, b, s1, 0.0f, mode, o1);
#pragma unroll
                for (int i = 0; i < 8; ++i) { packed[i] = o0[i]; packed[8 + i] = o1[i]; }
            }
            // The decoded values are in registers; now wait for the TMEM stage.
            if (lane == 0) ok = mbar_wait_bounded(&a_empty[as.s], as.ph ^ 1, p.err, p.wait_limit_ns) ? 1 : 0;
            ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
            if (!ok) return;
            tc_fence_after();
            tmem_st_32x32b_x16(tmem + lane_addr + (uint32_t)(C::A_COL0 + as.s * (BK / 2) + half * 16), packed);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&a_full[as.s]);
            xs.next<SS>();
            as.next<AS>();
        }
    }
}

template <int FMT, int BT, int ACC, int SS, int AS>
__global__ void __launch_bounds__(NUM_THREADS, 1) gemm_dq_kernel(const __grid_constant__ GemmParams p) {
    using C = Cfg<FMT, BT, ACC, SS, AS>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::OFF_BAR);
    uint64_t *x_full = bars;                 // [SS] TMA tx (x + codes)
    uint64_t *x_empty = x_full + SS;         // [SS] MMA commit
    uint64_t *a_full = x_empty + SS;         // [AS] 8 dequant warps
    uint64_t *a_empty = a_full + AS;         // [AS] MMA commit
    uint64_t *acc_full = a_empty + AS;       // [ACC] MMA commit
    uint64_t *acc_empty = acc_full + ACC;    // [ACC] 4 epilogue warps
    uint64_t *drain = acc_empty + ACC;       // [1] final MMA drain
    SmemCtl *ctl = reinterpret_cast<SmemCtl *>(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_mt = (p.M + BT - 1) / BT;
    const int n_ft = (p.N + 127) / 128;
    const int n_tiles = n_mt * n_ft;
    const int KB = (p.K + BK - 1) / BK;
    const int my_tiles = (int)blockIdx.x < n_tiles ? (n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    int *err = p.err;
    const uint64_t lim = p.wait_limit_ns;
    // Drains after an abort wait for copies / MMAs this CTA issued itself;
    // those finish in microseconds, so they get at least half a second even
    // when the pipeline limit is set very short.
    const uint64_t drain_lim = lim > 500000000ull ? lim : 500000000ull;

    if (threadIdx.x == 0) {
        for (int s = 0; s < SS; ++s) {
            mbar_init(&x_full[s], 1);
            mbar_init(&x_empty[s], 1);
        }
        for (int s = 0; s < AS; ++s) {
            mbar_init(&a_full[s], 8);
            mbar_init(&a_empty[s], 1);
        }
        for (int b = 0; b < ACC; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 4);
        }
        mbar_init(drain, 1);
        fence_mbar_init();
        tma_prefetch_desc(&p.tmap_x);
        tma_prefetch_desc(&p.tmap_w);
        if (FMT != FMT_BF16) tma_prefetch_desc(&p.tmap_s);
        if (FMT == FMT_FP8) tma_prefetch_desc(&p.tmap_f);
    }
    if (warp == 1) tmem_alloc(&ctl->tmem_base, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;

    if (warp == 0) {
        // ---------------- TMA producer: x tile + code tile ----------------
        if (lane == 0) {
            int last_phase[SS];
            for (int s = 0; s < SS; ++s) last_phase[s] = -1;
            const int wk_div = FMT == FMT_Q4 ? 2 : 1;  // the Q4 code map counts bytes (2 values)
            const uint32_t stage_tx = C::X_STAGE_BYTES + C::W_STAGE_BYTES +
                                      (FMT != FMT_BF16 ? 128 * 4 * p.sgrp : 0) + C::F_STAGE_BYTES;
            Ring xs;
            bool ok = true;
            for (int j = 0; j < my_tiles && ok; ++j) {
                const int tile = (int)blockIdx.x + j * (int)gridDim.x;
                const int mt = tile % n_mt, ft = tile / n_mt;
                for (int kb = 0; kb < KB; ++kb) {
                    if (!mbar_wait_bounded(&x_empty[xs.s], xs.ph ^ 1, err, lim)) { ok = false; break; }
                    mbar_arrive_expect_tx(&x_full[xs.s], stage_tx);
                    tma_load_2d(smem + xs.s * C::X_STAGE_BYTES, &p.tmap_x, &x_full[xs.s], kb * BK,
                                p.x_row + mt * BT);
                    tma_load_2d(smem + C::OFF_W + xs.s * C::W_STAGE_BYTES, &p.tmap_w, &x_full[xs.s],
                                kb * BK / wk_div, ft * 128);
                    if (FMT != FMT_BF16)
                        tma_load_2d(smem + C::OFF_S + xs.s * C::S_STAGE_BYTES, &p.tmap_s, &x_full[xs.s],
                                    ft * 128, (kb * BK) / p.group);
                    if (FMT == FMT_FP8)
                        tma_load_2d(smem + C::OFF_F + xs.s * C::F_STAGE_BYTES, &p.tmap_f, &x_full[xs.s],
                                    ft * 128, kb * 2);
                    last_phase[xs.s] = xs.ph;
                    xs.next<SS>();
                }
            }
            // Drain: every issued load has landed before smem can be released.
            for (int s = 0; s < SS; ++s)
                if (last_phase[s] >= 0) mbar_wait_bounded(&x_full[s], (uint32_t)last_phase[s], nullptr, drain_lim);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = idesc_bf16_f32(128, BT);
            bool ok = true;
            Ring xs, as, ab;
            for (int j = 0; j < my_tiles && ok; ++j) {
                if (!mbar_wait_bounded(&acc_empty[ab.s], ab.ph ^ 1, err, lim)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem + (uint32_t)(ab.s * BT);
                for (int kb = 0; kb < KB; ++kb) {
                    if (!mbar_wait_bounded(&x_full[xs.s], xs.ph, err, lim) ||
                        !mbar_wait_bounded(&a_full[as.s], as.ph, err, lim)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a_tmem = tmem + (uint32_t)(C::A_COL0 + as.s * (BK / 2));
                    const uint64_t b_desc = smem_desc_sw128(smem_u32(smem + xs.s * C::X_STAGE_BYTES));
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk)
                        mma_ts_f16(d_tmem, a_tmem + kk * 8, b_desc + (uint64_t)(kk * 2), idesc,
                                   (kb | kk) != 0);
                    mma_commit(&x_empty[xs.s]);
                    mma_commit(&a_empty[as.s]);
                    xs.next<SS>();
                    as.next<AS>();
                }
                if (!ok) break;
                mma_commit(&acc_full[ab.s]);
                ab.next<ACC>();
            }
            // Drain: all MMAs issued by this thread complete before TMEM is freed.
            mma_commit(drain);
            mbar_wait_bounded(drain, 0, nullptr, drain_lim);
        }
        __syncwarp();
    } else if (warp >= 4 && warp < 8) {
        // ---------------- epilogue ----------------
        // TMEM (thread = feature, 32 tokens) -> bias/GELU/gate -> smem staging
        // [32 tokens][128 features] -> 16-byte coalesced global stores, or
        // vector reductions (red.global.add) for the gated residual. Plain
        // stores keep the epilogue off the TMA queue, where the pipeline's
        // loads are waiting.
        const int q = warp - 4;
        const int et = threadIdx.x - 128;  // 0..127
        const bool leader = et == 0;
        int chunk_ctr = 0;
        const bool out_f32 = p.out_f32 != 0;
        const int esz = out_f32 ? 4 : 2;
        const int row_bytes = STG_COLS * esz;
        const int cpr = row_bytes / 16;  // 16-byte chunks per staged row
        Ring ab;
        for (int j = 0; j < my_tiles; ++j) {
            const int tile = (int)blockIdx.x + j * (int)gridDim.x;
            const int mt = tile % n_mt, ft = tile / n_mt;
            if (leader) ctl->epi_ok = mbar_wait_bounded(&acc_full[ab.s], ab.ph, err, lim) ? 1 : 0;
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
            const int nld = min(BT / 32, (p.M - m0 + 31) / 32);
            const uint32_t acc_addr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab.s * BT);
            for (int c = 0; c < nld; ++c) {
                uint32_t acc[32];
                tmem_ld_32x32b_x32(acc_addr + (uint32_t)(c * 32), acc);
                tmem_wait_ld();
                if (c == nld - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&acc_empty[ab.s]);
                }
                float2 v[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    float2 t = __fadd2_rn(make_float2(__uint_as_float(acc[2 * i]), __uint_as_float(acc[2 * i + 1])), bias2);
                    if (p.act == 1) t = gelu2(t);
                    v[i] = p.gate ? __fmul2_rn(t, gate2) : t;
                }
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int row0 = m0 + c * 32 + h * STG_ROWS;
                    if (row0 >= p.M) break;
                    uint8_t *stg = smem + C::OFF_STG + (chunk_ctr & 1) * C::STG_BYTES;
                    ++chunk_ctr;
                    if (out_f32) {
                        float *s32 = reinterpret_cast<float *>(stg) + q * 32 + lane;
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            s32[(2 * i) * STG_COLS] = v[h * 8 + i].x;
                            s32[(2 * i + 1) * STG_COLS] = v[h * 8 + i].y;
                        }
                    } else {
                        unsigned short *s16 = reinterpret_cast<unsigned short *>(stg) + q * 32 + lane;
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const uint32_t pk = pack_bf16x2(v[h * 8 + i]);
                            s16[(2 * i) * STG_COLS] = (unsigned short)(pk & 0xFFFFu);
                            s16[(2 * i + 1) * STG_COLS] = (unsigned short)(pk >> 16);
                        }
                    }
                    named_bar_sync(1, EPI_THREADS);
                    const int vals = 16 / esz;  // elements per 16-byte chunk
                    for (int id = et; id < STG_ROWS * cpr; id += EPI_THREADS) {
                        const int row = id / cpr, cc = id - row * cpr;
                        const int token = row0 + row;
                        const int f0 = ft * 128 + cc * vals;
                        if (token >= p.M || f0 >= p.N) continue;
                        const uint4 u = *reinterpret_cast<const uint4 *>(stg + row * row_bytes + cc * 16);
                        char *dst = reinterpret_cast<char *>(p.y) + (((int64_t)p.y_row + token) * p.N + f0) * esz;
                        if (!p.reduce) {
                            *reinterpret_cast<uint4 *>(dst) = u;
                        } else if (out_f32) {
                            asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst),
                                         "f"(__uint_as_float(u.x)), "f"(__uint_as_float(u.y)),
                                         "f"(__uint_as_float(u.z)), "f"(__uint_as_float(u.w))
                                         : "memory");
                        } else {
                            asm volatile("red.global.add.noftz.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(dst),
                                         "r"(u.x), "r"(u.y), "r"(u.z), "r"(u.w)
                                         : "memory");
                        }
                    }
                }
            }
            ab.next<ACC>();
        }
    } else if (warp >= 8) {
        dequant_role<FMT, BT, ACC, SS, AS>(p, smem, tmem, x_full, a_full, a_empty, warp, lane, KB, my_tiles);
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

// ---- host launcher --------------------------------------------------------
template <int FMT, int BT, int ACC, int SS, int AS>
static cudaError_t launch_t(const GemmParams &p, int num_sms, cudaStream_t st) {
    using C = Cfg<FMT, BT, ACC, SS, AS>;
    static bool attr_set = false;
    // Keep the footprint large enough that only one CTA fits per SM: each
    // CTA allocates all 512 TMEM columns.
    const int smem = C::SMEM_BYTES > 120 * 1024 ? C::SMEM_BYTES : 120 * 1024;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(gemm_dq_kernel<FMT, BT, ACC, SS, AS>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    const int n_tiles = ((p.M + BT - 1) / BT) * ((p.N + 127) / 128);
    const int grid = n_tiles < num_sms ? n_tiles : num_sms;
    gemm_dq_kernel<FMT, BT, ACC, SS, AS><<<grid, NUM_THREADS, smem, st>>>(p);
    return cudaGetLastError();
}

// Shared stages that fit next to the epilogue staging: each stage holds the
// x tile (BT*128 B) and the code tile (4, 8 or 16 KB), at most 8 stages.
constexpr int smem_stages(int fmt, int bt) {
    const int budget = 227 * 1024 - 1024 - 2 * STG_ROWS * STG_COLS * 4 - 512;
    const int w = 128 * (fmt == FMT_Q4 ? 32 : fmt == FMT_BF16 ? 128 : 64);
    const int side = fmt == FMT_Q4 ? 128 * 16 : fmt == FMT_BF16 ? 0 : 512 + (fmt == FMT_FP8 ? 256 : 0);
    const int stage = bt * BK * 2 + w + side;
    return budget / stage > 8 ? 8 : budget / stage;
}

// TMEM holds ACC*BT accumulator columns + AS*32 columns of decoded A.
template <int FMT>
static cudaError_t launch_fmt(int bt, const GemmParams &p, int num_sms, cudaStream_t st) {
    switch (bt) {
        case 128: return launch_t<FMT, 128, 2, smem_stages(FMT, 128), 8>(p, num_sms, st);
        case 192: return launch_t<FMT, 192, 2, smem_stages(FMT, 192), 4>(p, num_sms, st);
        case 256: return launch_t<FMT, 256, 1, smem_stages(FMT, 256), 8>(p, num_sms, st);
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
    // Measured on B200 (FP8 linears of the Wan2.1-1.3B chunk, M = 4680): the
    // widest token tile is fastest once there are enough tokens to fill it;
    // each decoded weight then feeds the most MMA columns.
    (void)N;
    (void)num_sms;
    if (M >= 1024) return 256;
    if (M >= 384) return 192;
    return 128;
}

}  // namespace lx2v
