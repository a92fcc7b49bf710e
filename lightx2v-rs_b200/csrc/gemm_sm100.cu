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
// Warp roles (24 warps, one persistent CTA per SM):
//   warp 0      TMA producer (x tile + code tile per stage)
//   warp 1      TMEM allocator and MMA issuer (one thread)
//   warps 4-7   epilogue: TMEM -> registers -> bias/GELU/gate -> smem staging
//               -> TMA store (or TMA reduce-add for the gated residual)
//   warps 8+    dequant: four warpgroups, each owns 16 of the 64 columns of
//               a k-block; thread = one weight row (TMEM lane)
// ACC accumulators (1 or 2) let the epilogue of tile j overlap the mainloop
// of tile j+1. Every mbarrier wait is bounded (ptx.cuh); on expiry the kernel
// records an error word, drains its own in-flight copies and MMAs, frees
// TMEM and returns.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <cstring>
#include "gemm_common.cuh"

namespace lx2v {


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
    static constexpr int OFF_W = SS * X_STAGE_BYTES;
    static constexpr int OFF_S = OFF_W + SS * W_STAGE_BYTES;
    static constexpr int OFF_F = OFF_S + SS * S_STAGE_BYTES;
    static constexpr int OFF_STG = (OFF_F + SS * F_STAGE_BYTES + 127) & ~127;
    static constexpr int OFF_BAR = OFF_STG + STG_TOTAL;
    static constexpr int NUM_BARS = 2 * SS + 2 * AS + 2 * ACC + 1;
    static constexpr int SMEM_BYTES = 1024 + OFF_BAR + NUM_BARS * 8 + 16;
    static_assert(X_STAGE_BYTES % 1024 == 0 && W_STAGE_BYTES % 1024 == 0, "swizzle atoms");
    static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
};

struct SmemCtl {
    uint32_t tmem_base;
    int epi_ok;
};

// Dequant warps: DQW warpgroups; thread = one weight row (TMEM lane) of the
// 128-row tile; warpgroup wg owns units [wg*U, wg*U + U) (16 columns each,
// U = 4/DQW) of every 64-wide k-block.
template <int FMT, int BT, int ACC, int SS, int AS, int DQW>
__device__ __forceinline__ void dequant_role(const GemmParams &p, uint8_t *smem, uint32_t tmem,
                                             uint64_t *x_full, uint64_t *a_full, uint64_t *a_empty,
                                             int warp, int lane, int KB, int my_tiles) {
    using C = Cfg<FMT, BT, ACC, SS, AS>;
    constexpr int U = 4 / DQW;
    const int q = warp & 3;
    const int u0 = ((warp - 8) >> 2) * U;
    const int r = q * 32 + lane;  // row within the 128-row tile
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    Ring xs, as;
    for (int j = 0; j < my_tiles; ++j) {
        for (int kb = 0; kb < KB; ++kb) {
            int ok = 1;
            if (lane == 0) ok = mbar_wait_bounded(&x_full[xs.s], xs.ph, p.err, p.wait_limit_ns) ? 1 : 0;
            ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
            if (!ok) return;
            uint32_t packed[8 * U];
            decode_units<FMT, U>(p, smem + C::OFF_W + xs.s * C::W_STAGE_BYTES, smem + C::OFF_S + xs.s * C::S_STAGE_BYTES,
                                 smem + C::OFF_F + xs.s * C::F_STAGE_BYTES, r, u0, packed);
            // The decoded values are in registers; now wait for the TMEM stage.
            if (lane == 0) ok = mbar_wait_bounded(&a_empty[as.s], as.ph ^ 1, p.err, p.wait_limit_ns) ? 1 : 0;
            ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
            if (!ok) return;
            tc_fence_after();
            const uint32_t ta = tmem + lane_addr + (uint32_t)(C::A_COL0 + as.s * (BK / 2) + u0 * 8);
#pragma unroll
            for (int u = 0; u < U; ++u) tmem_st_32x32b_x8(ta + u * 8, packed + 8 * u);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&a_full[as.s]);
            xs.next<SS>();
            as.next<AS>();
        }
    }
}

template <int FMT, int BT, int ACC, int SS, int AS, int DQW>
__global__ void __launch_bounds__(32 * (8 + 4 * DQW), 1) gemm_dq_kernel(const __grid_constant__ GemmParams p) {
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
            mbar_init(&a_full[s], 4 * DQW);
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
        const int q = warp - 4;
        const bool leader = threadIdx.x == 128;
        Ring ab;
        for (int j = 0; j < my_tiles; ++j) {
            const int tile = (int)blockIdx.x + j * (int)gridDim.x;
            const int mt = tile % n_mt, ft = tile / n_mt;
            if (leader) ctl->epi_ok = mbar_wait_bounded(&acc_full[ab.s], ab.ph, err, lim) ? 1 : 0;
            named_bar_sync(1, EPI_THREADS);
            if (!ctl->epi_ok) break;
            tc_fence_after();
            const uint32_t acc_addr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab.s * BT);
            uint64_t *rel_bar = &acc_empty[ab.s];
            epilogue_tile(p, acc_addr, BT, ft * 128, mt * BT, q, lane, smem + C::OFF_STG, [&] {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(rel_bar);
            });
            ab.next<ACC>();
        }
    } else if (warp >= 8) {
        dequant_role<FMT, BT, ACC, SS, AS, DQW>(p, smem, tmem, x_full, a_full, a_empty, warp, lane, KB, my_tiles);
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

// ---- host launcher --------------------------------------------------------
template <int FMT, int BT, int ACC, int SS, int AS, int DQW = 4>
static cudaError_t launch_t(const GemmParams &p, int num_sms, cudaStream_t st) {
    using C = Cfg<FMT, BT, ACC, SS, AS>;
    constexpr int NUM_THREADS = 32 * (8 + 4 * DQW);
    static std::atomic<int> attr_set_dev[LX2V_MAX_DEVICES];
    std::atomic<int> *slot = device_slot(attr_set_dev);
    // Keep the footprint large enough that only one CTA fits per SM: each
    // CTA allocates all 512 TMEM columns.
    const int smem = C::SMEM_BYTES > 120 * 1024 ? C::SMEM_BYTES : 120 * 1024;
    if (!slot || slot->load(std::memory_order_relaxed) == 0) {
        cudaError_t e = cudaFuncSetAttribute(gemm_dq_kernel<FMT, BT, ACC, SS, AS, DQW>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        if (slot) slot->store(1, std::memory_order_relaxed);
    }
    const int n_tiles = ((p.M + BT - 1) / BT) * ((p.N + 127) / 128);
    const int grid = n_tiles < num_sms ? n_tiles : num_sms;
    gemm_dq_kernel<FMT, BT, ACC, SS, AS, DQW><<<grid, NUM_THREADS, smem, st>>>(p);
    return cudaGetLastError();
}

// Shared stages that fit next to the epilogue staging: each stage holds the
// x tile (BT*128 B) and the code tile (4, 8 or 16 KB), at most 8 stages.
constexpr int smem_stages(int fmt, int bt) {
    const int budget = 227 * 1024 - 1024 - STG_TOTAL - 512;
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

int gemm_dq_token_tile(int M, int N, int K, int units, int feat_tile) {
    // Wave model of the persistent grid: `units` CTAs (or CTA pairs) each run
    // whole tiles of feat_tile features x bt tokens, so a launch takes
    // ceil(tiles / units) rounds of bt * (e * K + E) MMA-column time. Fitted on
    // B200 (FP8 linears of the Wan2.1-1.3B chunk at K = 1536 and 8960): the
    // 256-token tile has the cheapest k-loop (e = 1) but a single TMEM
    // accumulator, so its epilogue is exposed (E = 1190 k-columns); 192 tokens
    // keep two accumulators (E = 700) but pay the MMA thread's per-k-block
    // round trips on fewer columns (e = 1.42); 128 tokens: e = 1.9, E = 800.
    // Ties go to the wider tile. (M = 4680: QKV, out, FFN1, FFN2 -> 256.)
    const int cand[3] = {256, 192, 128};
    const double e[3] = {1.0, 1.42, 1.9}, E[3] = {1190.0, 700.0, 800.0};
    int best = 128;
    double best_cost = 0.0;
    for (int c = 0; c < 3; ++c) {
        const int bt = cand[c];
        if (c > 0 && M < bt / 2) continue;
        const long long tiles = (long long)((M + bt - 1) / bt) * ((N + feat_tile - 1) / feat_tile);
        const long long waves = (tiles + units - 1) / units;
        const double cost = (double)waves * bt * (e[c] * K + E[c]);
        if (c == 0 || cost < best_cost) {
            best = bt;
            best_cost = cost;
        }
    }
    return best;
}

}  // namespace lx2v
