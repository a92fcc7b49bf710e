// gemm_pair_sm100.cu — the quantized linear on a CTA pair (cta_group::2).
//
// Same computation as gemm_sm100.cu (Backend::linear and the fused gated
// residual, crates/lightx2v-core/src/backend.rs:199-212, 244-253), with the
// tile spread over a cluster of two CTAs on two SMs:
//   pair tile = 256 output features x BT tokens;
//   CTA r decodes weight rows [128 r, 128 r + 128) of the tile into its own
//   TMEM (A operand, 128 lanes per CTA) and TMA-loads tokens
//   [BT/2 r, BT/2 r + BT/2) of x into its own shared memory (B operand);
//   the leader CTA (rank 0) issues tcgen05.mma.cta_group::2 with M = 256,
//   N = BT, which reads A from both TMEMs and B from both shared memories and
//   leaves D = 128 features x BT tokens in each CTA's TMEM.
// Each SM thus loads half of the x tile per k-block: 24 KB of x + codes per
// 4.2 MFLOP instead of 40 KB, which is what lets the ring hold 8 stages and
// keep the tensor pipe fed from L2.
//
// Synchronisation (all waits bounded, ptx.cuh):
//   xb_full[s]  leader; both CTAs' x halves complete_tx on it (TMA
//               .cta_group::2, no multicast)
//   w_full[s]   each CTA; its own code / scale / flag tiles
//   x_empty[s]  each CTA; multicast tcgen05.commit from the leader once the
//               MMAs of the stage's k-block completed. It frees the smem
//               stage for the producer and, AS k-blocks later, the TMEM A
//               stage for the dequant warps (one commit per k-block).
//   a_full[a]   leader; 8 arrivals (the 4 warps of the dequant warpgroup that
//               owns the k-block, in both CTAs; remote for the peer). When the
//               two rings have the same depth (SS == AS) a_full is xb_full
//               itself (9 arrivals + the x bytes) and the MMA thread waits on
//               one barrier per k-block.
//   acc_full[b] each CTA; multicast commit
//   acc_empty[b] leader; 8 arrivals (4 epilogue warps x 2 CTAs)
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <cstring>
#include "gemm_common.cuh"

namespace lx2v {


template <int FMT, int BT, int ACC, int SS, int AS>
struct PairCfg {
    static constexpr int A_COL0 = ACC * BT;
    static_assert(A_COL0 + AS * (BK / 2) <= TMEM_COLS, "TMEM budget");
    static_assert(BT % 64 == 0 && BT <= 256, "pair token tile");
    static constexpr int XH_BYTES = (BT / 2) * BK * 2;  // this CTA's half of the x tile
    static constexpr int W_BYTES = WTile<FMT>::BYTES;
    static constexpr int S_BYTES = WTile<FMT>::S_BYTES;
    static constexpr int F_BYTES = WTile<FMT>::F_BYTES;
    static constexpr int OFF_W = SS * XH_BYTES;
    static constexpr int OFF_S = OFF_W + SS * W_BYTES;
    static constexpr int OFF_F = OFF_S + SS * S_BYTES;
    static constexpr int OFF_STG = (OFF_F + SS * F_BYTES + 127) & ~127;
    static constexpr int OFF_BAR = OFF_STG + STG_TOTAL;
    static constexpr int NUM_BARS = 3 * SS + AS + 2 * ACC + 1;
    static constexpr int SMEM_BYTES = 1024 + OFF_BAR + NUM_BARS * 8 + 16;
    static_assert(XH_BYTES % 1024 == 0 && W_BYTES % 1024 == 0, "swizzle atoms");
    static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
};

struct PairCtl {
    uint32_t tmem_base;
    int epi_ok;
};

template <int FMT, int BT, int ACC, int SS, int AS, int DQW, bool SK, int GRP>
__global__ void __launch_bounds__(32 * (8 + 4 * DQW), 1) gemm_pair_kernel(const __grid_constant__ GemmParams p) {
    using C = PairCfg<FMT, BT, ACC, SS, AS>;
    static_assert(SS >= AS, "an A stage is released through the x ring");
    static_assert(SS % DQW == 0, "each smem slot is read by one dequant warpgroup");
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::OFF_BAR);
    uint64_t *xb_full = bars;               // [SS]  leader: both x halves
    uint64_t *w_full = xb_full + SS;        // [SS]  own codes + side data
    uint64_t *x_empty = w_full + SS;        // [SS]  multicast commit: MMA of the stage done
    // With equal ring depths one barrier per stage carries both the x bytes
    // and the dequant arrivals, so the MMA thread waits once per k-block.
    constexpr bool MERGED = SS == AS;
    // GRP k-blocks form one MMA group: one ready wait and one commit per
    // group (the MMA thread's barrier round trips are what bounds the k-loop
    // on B200); data stays in 64-wide k-block stages.
    static_assert(SS % GRP == 0 && AS % GRP == 0, "k-block groups tile both rings");
    constexpr int NG = SS / GRP;   // group slots of xb_full / x_empty
    constexpr int NGA = AS / GRP;  // group slots of a_full (unmerged rings)
    uint64_t *a_full_sep = x_empty + SS;     // [AS]  leader: dequant warps of both CTAs (unmerged rings)
    uint64_t *a_full = MERGED ? xb_full : a_full_sep;
    uint64_t *acc_full = a_full_sep + AS;   // [ACC] multicast commit
    uint64_t *acc_empty = acc_full + ACC;   // [ACC] leader: 8 epilogue warps
    uint64_t *drain = acc_empty + ACC;      // [1]   leader: final MMA drain
    PairCtl *ctl = reinterpret_cast<PairCtl *>(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool lead = rank == 0;
    const int pair = (int)blockIdx.x >> 1, npairs = (int)gridDim.x >> 1;
    const int n_mt = (p.M + BT - 1) / BT;
    const int n_ft = (p.N + 255) / 256;
    const int n_tiles = n_mt * n_ft;
    const int KB = ((p.K + BK - 1) / BK) / GRP;  // groups per tile (the host keeps K a multiple of GRP k-blocks)
    PairWork work;
    work.KB = KB;
    work.pair = pair;
    work.npairs = npairs;
    work.my_tiles = pair < n_tiles ? (n_tiles - 1 - pair) / npairs + 1 : 0;
    work.sk = SK;
    const long long units = (long long)n_tiles * KB;
    work.init_split(n_tiles, 0);
    const int n_seg = work.count();
    const int total_gr = (int)work.total_kb();   // groups this pair runs, over all its segments
    const int total_kb = total_gr * GRP;          // k-blocks
    int *err = p.err;
    const uint64_t lim = p.wait_limit_ns;
    const uint64_t drain_lim = lim > 500000000ull ? lim : 500000000ull;

    if (threadIdx.x == 0) {
        for (int s = 0; s < SS; ++s) {
            mbar_init(&xb_full[s], MERGED ? 1 + 8 * GRP : 1);
            mbar_init(&w_full[s], 1);
            mbar_init(&x_empty[s], 1);
        }
        if (!MERGED)
            for (int s = 0; s < AS; ++s) mbar_init(&a_full[s], 8 * GRP);
        for (int b = 0; b < ACC; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 8);
        }
        mbar_init(drain, 1);
        fence_mbar_init();
        tma_prefetch_desc(&p.tmap_x);
        tma_prefetch_desc(&p.tmap_w);
        if (FMT != FMT_BF16) tma_prefetch_desc(&p.tmap_s);
        if (FMT == FMT_FP8) tma_prefetch_desc(&p.tmap_f);
    }
    if (warp == 1) tmem_alloc_pair(&ctl->tmem_base, TMEM_COLS);
    tc_fence_before();
    cluster_sync();  // barriers of both CTAs initialised, TMEM allocated
    tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;

    if (warp == 0) {
        // ---------------- TMA producer (both CTAs) ----------------
        if (lane == 0) {
            int last_phase[NG];
            for (int s = 0; s < NG; ++s) last_phase[s] = -1;
            const int wk_div = FMT == FMT_Q4 ? 2 : 1;
            const uint32_t w_tx = C::W_BYTES + (FMT != FMT_BF16 ? 128 * 4 * p.sgrp : 0) + C::F_BYTES;
            Ring gs;  // group slot
            bool ok = true;
            for (int j = 0; j < n_seg && ok; ++j) {
                int tile, kb0, kb1;
                work.seg(j, tile, kb0, kb1);
                const int mt = tile % n_mt, ft = tile / n_mt;
                const int row0 = ft * 256 + (int)rank * 128;
                const int xrow = p.x_row + mt * BT + (int)rank * (BT / 2);
                for (int gr = kb0; gr < kb1; ++gr) {
                    if (!mbar_wait_cluster_bounded(&x_empty[gs.s], gs.ph ^ 1, err, lim)) { ok = false; break; }
                    if (lead) mbar_arrive_expect_tx(&xb_full[gs.s], GRP * 2 * C::XH_BYTES);
                    const uint32_t xbar = mapa_shared(smem_u32(&xb_full[gs.s]), 0);
#pragma unroll
                    for (int h = 0; h < GRP; ++h) {
                        const int kb = gr * GRP + h;
                        const int s = gs.s * GRP + h;  // data stage slot
                        mbar_arrive_expect_tx(&w_full[s], w_tx);
                        tma_load_2d_pair(smem + s * C::XH_BYTES, &p.tmap_x, xbar, kb * BK, xrow);
                        tma_load_2d(smem + C::OFF_W + s * C::W_BYTES, &p.tmap_w, &w_full[s], kb * BK / wk_div, row0);
                        if (FMT != FMT_BF16)
                            tma_load_2d(smem + C::OFF_S + s * C::S_BYTES, &p.tmap_s, &w_full[s], row0,
                                        (kb * BK) / p.group);
                        if (FMT == FMT_FP8)
                            tma_load_2d(smem + C::OFF_F + s * C::F_BYTES, &p.tmap_f, &w_full[s], row0, kb * 2);
                    }
                    last_phase[gs.s] = gs.ph;
                    gs.next<NG>();
                }
            }
            // Drain: a group's loads have landed once its codes arrived and the
            // leader's MMA released it (x halves are counted on the leader).
            for (int g2 = 0; g2 < NG; ++g2)
                if (last_phase[g2] >= 0) {
                    for (int h = 0; h < GRP; ++h)
                        mbar_wait_bounded(&w_full[g2 * GRP + h], (uint32_t)last_phase[g2], nullptr, drain_lim);
                    mbar_wait_cluster_bounded(&x_empty[g2], (uint32_t)last_phase[g2], nullptr, drain_lim);
                }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer (leader CTA) ----------------
        // One wait per barrier per k-block, right before its MMAs: the MMAs
        // already issued keep the tensor pipe busy meanwhile. (Non-blocking
        // look-ahead tests of the next stage measured slower on B200: each
        // barrier access is a ~150-cycle round trip on this thread's path.)
        if (lane == 0 && lead) {
            const uint32_t idesc = idesc_bf16_f32(256, BT);
            bool ok = true;
            Ring xs, as, ab, ag;  // xs: group slot (NG), as: A stage (AS, per k-block), ag: A group slot (NGA)
            bool x_ready = total_kb > 0 && mbar_wait_cluster_bounded(&xb_full[0], 0, err, lim);
            bool a_ready = x_ready && (MERGED || mbar_wait_cluster_bounded(&a_full[0], 0, err, lim));
            ok = total_gr == 0 || (x_ready && a_ready);
            int i = 0;
            for (int j = 0; j < n_seg && ok; ++j) {
                int tile, kb0, kb1;
                work.seg(j, tile, kb0, kb1);
                if (!mbar_wait_cluster_bounded(&acc_empty[ab.s], ab.ph ^ 1, err, lim)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem + (uint32_t)(ab.s * BT);
                for (int kb = kb0; kb < kb1; ++kb, ++i) {
                    if (i > 0 && (!mbar_wait_cluster_bounded(&xb_full[xs.s], xs.ph, err, lim) ||
                                  (!MERGED && !mbar_wait_cluster_bounded(&a_full[ag.s], ag.ph, err, lim)))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int h = 0; h < GRP; ++h) {
                        const uint32_t a_tmem = tmem + (uint32_t)(C::A_COL0 + as.s * (BK / 2));
                        const uint64_t b_desc = smem_desc_sw128(smem_u32(smem + (xs.s * GRP + h) * C::XH_BYTES));
#pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk)
                            mma_ts_f16_pair(d_tmem, a_tmem + kk * 8, b_desc + (uint64_t)(kk * 2), idesc,
                                            (kb != kb0 || h != 0 || kk != 0) ? 1u : 0u);
                        as.next<AS>();
                    }
                    mma_commit_pair(&x_empty[xs.s], 0x3);
                    if (kb == kb1 - 1) mma_commit_pair(&acc_full[ab.s], 0x3);
                    xs.next<NG>();
                    ag.next<NGA>();
                }
                if (!ok) break;
                ab.next<ACC>();
            }
            mma_commit_pair(drain, 0x1);
            mbar_wait_bounded(drain, 0, nullptr, drain_lim);
        }
        __syncwarp();
    } else if (warp >= 4 && warp < 8) {
        // ---------------- epilogue (both CTAs) ----------------
        const int q = warp - 4;
        const bool leader_thread = threadIdx.x == 128;
        Ring ab;
        const int64_t part_floats = (int64_t)128 * BT;  // one CTA's partial tile
        for (int j = 0; j < n_seg; ++j) {
            int tile, kb0, kb1;
            work.seg(j, tile, kb0, kb1);
            const int mt = tile % n_mt, ft = tile / n_mt;
            PartialIO io;
            int n_add = 0;
            if (!SK) {
            } else if (kb0 > 0) {
                // the tail of a split tile: its owner adds it later
                io.write = p.partials + (int64_t)(pair * 2 + (int)rank) * part_floats;
            } else if (kb1 < KB) {
                // the head of a split tile: the pairs after this one hold the rest
                const long long tile_end = (long long)(tile + 1) * KB;
                while (pair + 1 + n_add < npairs && units * (pair + 1 + n_add) / npairs < tile_end) ++n_add;
            }
            if (leader_thread) {
                bool ok = mbar_wait_cluster_bounded(&acc_full[ab.s], ab.ph, err, lim);
                for (int a = 0; SK && a < n_add && ok; ++a)
                    ok = flag_wait_bounded(p.flags + (pair + 1 + a) * 2 + (int)rank, p.epoch, err, lim);
                ctl->epi_ok = ok ? 1 : 0;
            }
            named_bar_sync(1, EPI_THREADS);
            if (!ctl->epi_ok) break;
            tc_fence_after();
            if (SK && n_add > 0) {
                asm volatile("fence.acq_rel.gpu;" ::: "memory");
                io.add = p.partials + (int64_t)((pair + 1) * 2 + (int)rank) * part_floats;
                io.n_add = n_add;
                io.add_stride = 2 * part_floats;
            }
            const uint32_t acc_addr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab.s * BT);
            const uint32_t rel = mapa_shared(smem_u32(&acc_empty[ab.s]), 0);
            epilogue_tile<SK>(p, acc_addr, BT, ft * 256 + (int)rank * 128, mt * BT, q, lane, smem + C::OFF_STG,
                          [&] {
                              tc_fence_before();
                              __syncwarp();
                              if (lane == 0) mbar_arrive_cluster(rel);
                          }, io);
            if (SK && io.write) {
                __threadfence();
                named_bar_sync(1, EPI_THREADS);
                if (leader_thread) flag_publish(p.flags + pair * 2 + (int)rank, p.epoch);
            }
            if (SK && n_add > 0) {
                // every epilogue thread has read the tail pairs' partials:
                // clear their flags, so that a later launch with the same
                // epoch (a replayed CUDA graph) waits for fresh partials
                named_bar_sync(1, EPI_THREADS);
                if (leader_thread)
                    for (int a = 0; a < n_add; ++a) flag_clear(p.flags + (pair + 1 + a) * 2 + (int)rank);
            }
            ab.next<ACC>();
        }
    } else if (warp >= 8) {
        // ---------------- dequant (both CTAs) ----------------
        // Warpgroup g takes whole k-blocks i = g, g + DQW, ... of the pair's
        // sequence; thread r decodes weight row r (64 values) and writes them
        // to A stage i % AS of its CTA's TMEM. The A stage is free once the
        // MMA of k-block i - AS has completed, which the x ring's empty
        // barrier of that k-block records.
        const int g = (warp - 8) >> 2;
        const int q = warp & 3;
        const int r = q * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
        for (int i = g; i < total_kb; i += DQW) {
            const int s = i % SS;
            const uint32_t ph = (uint32_t)(i / SS) & 1u;
            const int a = i % AS;
            int w = 1;
            if (lane == 0) {
                w = mbar_wait_bounded(&w_full[s], ph, err, lim) ? 1 : 0;
                if (w && i >= AS) {
                    const int e = (i - AS) / GRP;  // the group whose MMAs free this A stage
                    w = mbar_wait_cluster_bounded(&x_empty[e % NG], (uint32_t)(e / NG) & 1u, err, lim) ? 1 : 0;
                }
            }
            w = __shfl_sync(0xFFFFFFFFu, w, 0);
            if (!w) break;
            tc_fence_after();
            const uint32_t ta = tmem + lane_addr + (uint32_t)(C::A_COL0 + a * (BK / 2));
            const uint8_t *wst = smem + C::OFF_W + s * C::W_BYTES;
            const uint8_t *sst = smem + C::OFF_S + s * C::S_BYTES;
            const uint8_t *fst = smem + C::OFF_F + s * C::F_BYTES;
            {
                uint32_t packed[32];
                decode_units<FMT, 4>(p, wst, sst, fst, r, 0, packed);
                tmem_st_32x32b_x16(ta, *reinterpret_cast<uint32_t(*)[16]>(packed));
                tmem_st_32x32b_x16(ta + 16u, *reinterpret_cast<uint32_t(*)[16]>(packed + 16));
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0)
                mbar_arrive_cluster(mapa_shared(smem_u32(&a_full[MERGED ? (i / GRP) % NG : (i / GRP) % NGA]), 0));
        }
    }

    tc_fence_before();
    cluster_sync();  // the leader's MMAs and both epilogues are done with both TMEMs
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem, TMEM_COLS);
}

// ---- host launcher --------------------------------------------------------
constexpr int cmin(int a, int b) { return a < b ? a : b; }

constexpr int pair_stages(int fmt, int bt) {
    const int budget = 227 * 1024 - 1024 - STG_TOTAL - 512;
    const int w = 128 * (fmt == FMT_Q4 ? 32 : fmt == FMT_BF16 ? 128 : 64);
    const int side = fmt == FMT_Q4 ? 128 * 16 : fmt == FMT_BF16 ? 0 : 512 + (fmt == FMT_FP8 ? 256 : 0);
    const int stage = (bt / 2) * BK * 2 + w + side;
    // A multiple of the four dequant warpgroups: each ring slot is then read
    // by one warpgroup only, which has waited out the slot's previous phase
    // itself (a parity wait must never run a whole phase ahead).
    const int n = budget / stage > 8 ? 8 : budget / stage;
    return n - n % 4;
}

template <int FMT, int BT, int ACC, int SS, int AS, bool SK, int GRP, int DQW = 4>
static cudaError_t pair_launch_sk(const GemmParams &p, int num_sms, cudaStream_t st) {
    using C = PairCfg<FMT, BT, ACC, SS, AS>;
    auto kern = gemm_pair_kernel<FMT, BT, ACC, SS, AS, DQW, SK, GRP>;
    constexpr int PAIR_THREADS = 32 * (8 + 4 * DQW);
    static std::atomic<int> max_pairs_dev[LX2V_MAX_DEVICES];
    std::atomic<int> *slot = device_slot(max_pairs_dev);
    int max_pairs = slot ? slot->load(std::memory_order_relaxed) : 0;
    const int smem = C::SMEM_BYTES > 120 * 1024 ? C::SMEM_BYTES : 120 * 1024;
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof cfg);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(PAIR_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (max_pairs == 0) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        cfg.gridDim = dim3(2 * (num_sms / 2));
        int clusters = 0;
        e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
        if (e != cudaSuccess) return e;
        max_pairs = clusters > 0 ? clusters : 1;
        if (slot) slot->store(max_pairs, std::memory_order_relaxed);
    }
    const int n_tiles = ((p.M + BT - 1) / BT) * ((p.N + 255) / 256);
    // stream-K: every pair gets at least one k-block (the host checked
    // n_tiles * KB >= pairs)
    const long long work = SK ? (long long)n_tiles * (((p.K + BK - 1) / BK) / GRP) : n_tiles;
    const int pairs = work < max_pairs ? (int)work : max_pairs;
    cfg.gridDim = dim3(2 * pairs);
    return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int FMT, int BT, int ACC, int SS, int AS>
static cudaError_t pair_launch_t(const GemmParams &p, int num_sms, cudaStream_t st) {
    if constexpr (SS % 2 == 0 && AS % 2 == 0) {
        if (p.kgroup == 2)
            return p.streamk ? pair_launch_sk<FMT, BT, ACC, SS, AS, true, 2>(p, num_sms, st)
                             : pair_launch_sk<FMT, BT, ACC, SS, AS, false, 2>(p, num_sms, st);
    }
    return p.streamk ? pair_launch_sk<FMT, BT, ACC, SS, AS, true, 1>(p, num_sms, st)
                     : pair_launch_sk<FMT, BT, ACC, SS, AS, false, 1>(p, num_sms, st);
}

template <int FMT>
static cudaError_t pair_launch_fmt(int bt, const GemmParams &p, int num_sms, cudaStream_t st) {
    switch (bt) {
        case 128: return pair_launch_t<FMT, 128, 2, pair_stages(FMT, 128), cmin(8, pair_stages(FMT, 128))>(p, num_sms, st);
        case 192: return pair_launch_t<FMT, 192, 2, pair_stages(FMT, 192), cmin(4, pair_stages(FMT, 192))>(p, num_sms, st);
        case 256: return pair_launch_t<FMT, 256, 1, pair_stages(FMT, 256), cmin(8, pair_stages(FMT, 256))>(p, num_sms, st);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t gemm_pair_launch(int fmt, int bt, const GemmParams &p, int num_sms, cudaStream_t st) {
    switch (fmt) {
        case FMT_Q8: return pair_launch_fmt<FMT_Q8>(bt, p, num_sms, st);
        case FMT_Q4: return pair_launch_fmt<FMT_Q4>(bt, p, num_sms, st);
        case FMT_FP8: return pair_launch_fmt<FMT_FP8>(bt, p, num_sms, st);
        default: return pair_launch_fmt<FMT_BF16>(bt, p, num_sms, st);
    }
}

}  // namespace lx2v
