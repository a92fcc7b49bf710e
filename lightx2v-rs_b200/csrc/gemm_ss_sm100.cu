// gemm_ss_sm100.cu — second pass of the two-pass linear: y = act(x W^T + b)
// (or h += gate * act(x W^T + b)) with W already decoded to a bf16 [N][K]
// array (dequant_bf16_kernel, or a bf16 weight as uploaded). Same result as
// the one-pass kernels (Backend::linear and the fused gated residual,
// crates/lightx2v-core/src/backend.rs:199-212, 244-253): both multiply the
// same bf16 operands with f32 accumulation.
//
// Why two passes: at thousands of tokens each weight element is used by
// every token tile, so decoding it once per call (an HBM-bound pass over
// N x K) and then running a GEMM whose operands both come from shared memory
// costs less than decoding it again for every token tile inside the GEMM,
// where the decode warps share the SM with the MMA-issuing thread.
//
// Tile: a cluster of two CTAs on two SMs computes 256 output features x BT
// tokens with tcgen05.mma.cta_group::2.kind::f16 (M = 256, N = BT, K = 16):
// CTA r TMA-loads weight rows [128 r, 128 r + 128) of the tile (A) and tokens
// [BT/2 r, BT/2 r + BT/2) of x (B) into its own shared memory, both 128-byte
// swizzled K-major; the leader issues the MMAs. Accumulators: ACC buffers of
// BT TMEM columns, so the epilogue of one tile overlaps the k-loop of the
// next. Persistent grid of CTA pairs, tiles strided over pairs, feature tile
// fastest (pairs running at the same time share x tiles; measured 3 % faster
// than token tile fastest on the 1.3B chunk's QKV and FFN2).
//
// Warp roles (384 threads per CTA): warp 0 TMA producer (both CTAs), warp 1
// MMA issuer (leader CTA) and TMEM allocation, warps 4-11 epilogue (both
// CTAs): warp w reads TMEM lanes 32 (w % 4) .. + 31 of token columns
// [BT/2 h, BT/2 h + BT/2), h = (w - 4) / 4. Per 32-token chunk a warp puts
// its 32 features x 32 tokens into its own shared-memory box and one lane
// writes the box with a TMA tensor store (a TMA reduce-add for the f32
// gated residual): stores of two bytes per thread from registers measured
// ~6 us of a ~8 us tile epilogue, as long as the k-loop of a K = 1536 tile.
//
// Synchronisation (all waits bounded, ptx.cuh), per group of GRP k-blocks:
//   full[g]      leader; 1 arrival (the leader producer's expect_tx) plus the
//                A and x bytes of both CTAs (TMA .cta_group::2, no multicast)
//   empty[g]     each CTA; multicast tcgen05.commit once the group's MMAs
//                completed: frees both CTAs' stages of the group
//   acc_full[b]  each CTA; multicast commit after a tile's last group
//   acc_empty[b] leader; 16 arrivals (8 epilogue warps x 2 CTAs)
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <cstring>
#include "gemm_common.cuh"

namespace lx2v {

constexpr int SS_EPI_WARPS = 8;
constexpr int SS_STG_BOX = 32 * 32 * 4;                   // bytes of one warp's staging box
constexpr int SS_STG_BYTES = SS_EPI_WARPS * SS_STG_BOX;

template <int BT, int ACC, int SS>
struct SsCfg {
    static constexpr int XH_BYTES = (BT / 2) * BK * 2;  // this CTA's half of the x tile
    static constexpr int A_BYTES = 128 * BK * 2;        // this CTA's 128 weight rows
    static constexpr int OFF_A = SS * XH_BYTES;
    static constexpr int OFF_STG = OFF_A + SS * A_BYTES;      // per epilogue warp: one 32 x 32 f32 box
    static constexpr int OFF_BAR = OFF_STG + SS_STG_BYTES;
    static constexpr int NUM_BARS = 2 * SS + 2 * ACC + 1;
    static constexpr int SMEM_BYTES = 1024 + OFF_BAR + NUM_BARS * 8 + 16;
    static_assert(ACC * BT <= TMEM_COLS, "TMEM budget");
    static_assert(BT % 64 == 0 && BT <= 256, "pair token tile");
    static_assert(XH_BYTES % 1024 == 0 && A_BYTES % 1024 == 0, "swizzle atoms");
    static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
};

constexpr int SS_THREADS = 32 * (4 + SS_EPI_WARPS);

struct SsCtl {
    uint32_t tmem_base;
};

// Stream-K partial tiles of one epilogue warp (GemmParams::streamk). A
// partial tile is this CTA's raw f32 accumulator, [token column][128
// features], so a warp's accesses for one token are 128 contiguous bytes.
struct SkIO {
    float *write = nullptr;      // non-null: store the raw accumulator here, nothing else
    const float *add = nullptr;  // add n_add partial tiles from here (stride apart) before the epilogue
    int n_add = 0;
    int64_t stride = 0;
};

// One 32-token chunk of the epilogue: v[j] = the f32 accumulator of token
// tok0 + j (tile column col0 + j) for this thread's feature f (feature fl of
// the CTA's 128). Bias, GELU and gate in f32 exactly as epilogue_tile does
// them; each store of a warp covers one token's 32 consecutive features.
template <bool SK>
__device__ __forceinline__ void store_chunk(const GemmParams &p, const uint32_t (&v)[32], int tok0, int f, bool fok,
                                           float2 bias2, float2 gate2, const SkIO &io, int col0, int fl,
                                           uint8_t *stg, int lane) {
    const int nt = min(32, p.M - tok0);
    const int64_t n = p.N;
    const int64_t off0 = ((int64_t)p.y_row + tok0) * n + f;
    float acc[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) acc[j] = __uint_as_float(v[j]);
    if (SK) {
        if (io.write) {
            float *dst = io.write + (int64_t)col0 * 128 + fl;
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (j < nt) __stcg(dst + j * 128, acc[j]);
            __syncwarp();
            return;
        }
        for (int part = 0; part < io.n_add; ++part) {
            const float *src = io.add + part * io.stride + (int64_t)col0 * 128 + fl;
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (j < nt) acc[j] += __ldcg(src + j * 128);
        }
    }
    float o[32];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        float2 t = __fadd2_rn(make_float2(acc[2 * i], acc[2 * i + 1]), bias2);
        if (p.act == 1) t = gelu2(t);
        if (p.gate) t = __fmul2_rn(t, gate2);
        o[2 * i] = t.x;
        o[2 * i + 1] = t.y;
    }
    if (p.tma_y) {
        // [32 tokens][32 features] row-major box, as the tensor map reads it
        if (lane == 0) bulk_wait_read<0>();  // the previous box has been read out
        __syncwarp();
        if (p.out_f32) {
            float *b = reinterpret_cast<float *>(stg);
#pragma unroll
            for (int j = 0; j < 32; ++j) b[j * 32 + lane] = o[j];
        } else {
            __nv_bfloat16 *b = reinterpret_cast<__nv_bfloat16 *>(stg);
#pragma unroll
            for (int j = 0; j < 32; ++j) b[j * 32 + lane] = __float2bfloat16_rn(o[j]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        const int c0 = f - lane, c1 = p.y_row + tok0;  // c0: this warp's first feature, a multiple of 32
        if (lane == 0 && c0 < p.N) {
            // rows past y_row + M and columns past N fall outside the map and are not written
            if (p.reduce) tma_reduce_add_2d(&p.tmap_y, stg, c0, c1);
            else tma_store_2d(&p.tmap_y, stg, c0, c1);
            bulk_commit();
        }
        __syncwarp();
        return;
    }
    if (p.out_f32) {
        float *dst = reinterpret_cast<float *>(p.y) + off0;
        if (!p.reduce) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (fok && j < nt) dst[j * n] = o[j];
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (fok && j < nt)
                    asm volatile("red.global.add.f32 [%0], %1;" ::"l"(dst + j * n), "f"(o[j]) : "memory");
        }
    } else {
        __nv_bfloat16 *dst = reinterpret_cast<__nv_bfloat16 *>(p.y) + off0;
        if (!p.reduce) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (fok && j < nt) dst[j * n] = __float2bfloat16_rn(o[j]);
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (fok && j < nt) {
                    const __nv_bfloat16 h = __float2bfloat16_rn(o[j]);
                    asm volatile("red.global.add.noftz.bf16 [%0], %1;" ::"l"(dst + j * n),
                                 "h"(*reinterpret_cast<const unsigned short *>(&h))
                                 : "memory");
                }
        }
    }
    __syncwarp();  // the next tcgen05 instruction is warp-collective
}

// Epilogue of `ntok` accumulator columns from `acc_addr` (this thread: TMEM
// lane = output feature f; tokens m0 .., m0 < M) without a staging copy: the
// next 32-column TMEM load is in flight while a chunk is stored. `release`
// runs once the last load has completed.
template <bool SK, typename Release>
__device__ __forceinline__ void epilogue_direct(const GemmParams &p, uint32_t acc_addr, int ntok, int f, int m0,
                                                Release release, const SkIO &io, int col0, int fl, uint8_t *stg,
                                                int lane, bool with_bias) {
    const bool fok = f < p.N;
    float bias_f = 0.0f, gate_f = 1.0f;
    if (fok) {
        if (p.bias && with_bias) bias_f = p.bias_f32 ? reinterpret_cast<const float *>(p.bias)[f]
                                        : __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p.bias)[f]);
        if (p.gate) gate_f = p.gate_f32 ? reinterpret_cast<const float *>(p.gate)[f]
                                        : __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p.gate)[f]);
    }
    const float2 bias2 = make_float2(bias_f, bias_f), gate2 = make_float2(gate_f, gate_f);
    const int nld = min(ntok / 32, (p.M - m0 + 31) / 32);
    uint32_t a[32], b[32];
    tmem_ld_32x32b_x32(acc_addr, a);
    for (int c = 0; c < nld; c += 2) {
        tmem_wait_ld_regs(a);
        if (c + 1 < nld) tmem_ld_32x32b_x32(acc_addr + (uint32_t)((c + 1) * 32), b);
        else release();
        store_chunk<SK>(p, a, m0 + c * 32, f, fok, bias2, gate2, io, col0 + c * 32, fl, stg, lane);
        if (c + 1 < nld) {
            tmem_wait_ld_regs(b);
            if (c + 2 < nld) tmem_ld_32x32b_x32(acc_addr + (uint32_t)((c + 2) * 32), a);
            else release();
            store_chunk<SK>(p, b, m0 + (c + 1) * 32, f, fok, bias2, gate2, io, col0 + (c + 1) * 32, fl, stg, lane);
        }
    }
}

template <int BT, int ACC, int SS, int GRP, bool SK>
__global__ void __launch_bounds__(SS_THREADS, 1) gemm_ss_pair_kernel(const __grid_constant__ GemmParams p) {
    using C = SsCfg<BT, ACC, SS>;
    static_assert(SS % GRP == 0, "k-block groups tile the ring");
    constexpr int NG = SS / GRP;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::OFF_BAR);
    uint64_t *full = bars;                  // [NG]
    uint64_t *empty = full + NG;            // [NG]
    uint64_t *acc_full = empty + NG;        // [ACC]
    uint64_t *acc_empty = acc_full + ACC;   // [ACC]
    uint64_t *drain = acc_empty + ACC;      // [1]
    SsCtl *ctl = reinterpret_cast<SsCtl *>(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool lead = rank == 0;
    const int pair = (int)blockIdx.x >> 1, npairs = (int)gridDim.x >> 1;
    const int n_mt = (p.M + BT - 1) / BT;
    const int n_ft = (p.N + 255) / 256;
    const int n_tiles = n_mt * n_ft;
    const int KG = ((p.K + BK - 1) / BK) / GRP;  // groups per tile (the host keeps K a multiple of GRP k-blocks)
    PairWork work;
    work.KB = KG;
    work.pair = pair;
    work.npairs = npairs;
    work.ks = !SK && p.ksplit > 1 ? p.ksplit : 1;
    work.n_tiles = n_tiles;
    const int n_items = n_tiles * work.ks;
    work.my_tiles = pair < n_items ? (n_items - 1 - pair) / npairs + 1 : 0;
    work.sk = SK;
    // stream-K: full waves of whole tiles first, the rest split
    work.init_split(n_tiles, (n_tiles / npairs) * npairs);
    const int n_seg = work.count();
    int *err = p.err;
    const uint64_t lim = p.wait_limit_ns;
    const uint64_t drain_lim = lim > 500000000ull ? lim : 500000000ull;

    if (threadIdx.x == 0) {
        for (int g = 0; g < NG; ++g) {
            mbar_init(&full[g], 1);
            mbar_init(&empty[g], 1);
        }
        for (int b = 0; b < ACC; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 2 * SS_EPI_WARPS);
        }
        mbar_init(drain, 1);
        fence_mbar_init();
        tma_prefetch_desc(&p.tmap_x);
        tma_prefetch_desc(&p.tmap_w);
    }
    if (warp == 1) tmem_alloc_pair(&ctl->tmem_base, TMEM_COLS);
    tc_fence_before();
    cluster_sync();  // barriers of both CTAs initialised, TMEM allocated
    tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;
    // Launched as a programmatic dependent: everything above overlapped the
    // previous kernel (the weight decode); from here on this kernel reads its
    // output (and x, y written earlier in the stream). Once past the wait,
    // the next kernel in the stream may start (the next linear's decode,
    // which touches nothing this one reads).
    griddep_wait();
    griddep_launch_dependents();

    if (warp == 0) {
        // ---------------- TMA producer (both CTAs) ----------------
        if (lane == 0) {
            int last_phase[NG];
            for (int g = 0; g < NG; ++g) last_phase[g] = -1;
            constexpr uint32_t tx = GRP * 2 * (C::XH_BYTES + C::A_BYTES);
            Ring gs;
            bool ok = true;
            for (int j = 0; j < n_seg && ok; ++j) {
                int t, kb0, kb1;
                work.seg(j, t, kb0, kb1);
                const int mt = t / n_ft, ft = t % n_ft;
                const int row0 = ft * 256 + (int)rank * 128;
                const int xrow = p.x_row + mt * BT + (int)rank * (BT / 2);
                for (int gr = kb0; gr < kb1; ++gr) {
                    if (!mbar_wait_cluster_bounded(&empty[gs.s], gs.ph ^ 1, err, lim)) { ok = false; break; }
                    if (lead) mbar_arrive_expect_tx(&full[gs.s], tx);
                    const uint32_t fbar = mapa_shared(smem_u32(&full[gs.s]), 0);
#pragma unroll
                    for (int h = 0; h < GRP; ++h) {
                        const int kb = gr * GRP + h;
                        const int s = gs.s * GRP + h;
                        tma_load_2d_pair(smem + s * C::XH_BYTES, &p.tmap_x, fbar, kb * BK, xrow);
                        tma_load_2d_pair(smem + C::OFF_A + s * C::A_BYTES, &p.tmap_w, fbar, kb * BK, row0);
                    }
                    last_phase[gs.s] = gs.ph;
                    gs.next<NG>();
                }
            }
            // Drain: a group's loads have landed once the leader's MMAs
            // released it.
            for (int g = 0; g < NG; ++g)
                if (last_phase[g] >= 0) mbar_wait_cluster_bounded(&empty[g], (uint32_t)last_phase[g], nullptr, drain_lim);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer (leader CTA) ----------------
        if (lane == 0 && lead) {
            const uint32_t idesc = idesc_bf16_f32(256, BT);
            Ring gs, ab;
            bool ok = true;
            for (int j = 0; j < n_seg && ok; ++j) {
                int t, kb0, kb1;
                work.seg(j, t, kb0, kb1);
                if (!mbar_wait_cluster_bounded(&acc_empty[ab.s], ab.ph ^ 1, err, lim)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem + (uint32_t)(ab.s * BT);
                for (int gr = kb0; gr < kb1; ++gr) {
                    if (!mbar_wait_cluster_bounded(&full[gs.s], gs.ph, err, lim)) { ok = false; break; }
                    tc_fence_after();
#pragma unroll
                    for (int h = 0; h < GRP; ++h) {
                        const int s = gs.s * GRP + h;
                        const uint64_t a_desc = smem_desc_sw128(smem_u32(smem + C::OFF_A + s * C::A_BYTES));
                        const uint64_t b_desc = smem_desc_sw128(smem_u32(smem + s * C::XH_BYTES));
#pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk)
                            mma_ss_f16_pair(d_tmem, a_desc + (uint64_t)(kk * 2), b_desc + (uint64_t)(kk * 2), idesc,
                                            (gr != kb0 || h != 0 || kk != 0) ? 1u : 0u);
                    }
                    mma_commit_pair(&empty[gs.s], 0x3);
                    if (gr == kb1 - 1) mma_commit_pair(&acc_full[ab.s], 0x3);
                    gs.next<NG>();
                }
                ab.next<ACC>();
            }
            mma_commit_pair(drain, 0x1);
            mbar_wait_bounded(drain, 0, nullptr, drain_lim);
        }
        __syncwarp();
    } else if (warp >= 4) {
        // ---------------- epilogue (both CTAs) ----------------
        const int q = warp & 3, half = (warp - 4) >> 2, wi = warp - 4;
        const int64_t part_floats = (int64_t)128 * BT;  // one CTA's partial tile
        Ring ab;
        for (int j = 0; j < n_seg; ++j) {
            int t, kb0, kb1;
            work.seg(j, t, kb0, kb1);
            const int mt = t / n_ft, ft = t % n_ft;
            SkIO io;
            int n_add = 0;
            if (!SK) {
            } else if (kb0 > 0) {
                // the tail of a split tile: the pair holding its head adds it
                io.write = p.partials + (int64_t)(pair * 2 + (int)rank) * part_floats;
            } else if (kb1 < KG) {
                // the head of a split tile: the pairs after this one hold the rest
                const long long tile_end = (long long)(t + 1) * KG;
                while (pair + 1 + n_add < npairs && work.split_start(n_tiles, pair + 1 + n_add) < tile_end) ++n_add;
            }
            int ok = 1;
            if (lane == 0) {
                ok = mbar_wait_cluster_bounded(&acc_full[ab.s], ab.ph, err, lim) ? 1 : 0;
                // each warp waits for the same warp of the tail pairs: they
                // wrote exactly the lanes and columns it reads
                for (int a = 0; SK && a < n_add && ok; ++a)
                    ok = flag_wait_bounded(p.flags + ((pair + 1 + a) * 2 + (int)rank) * SS_EPI_WARPS + wi, p.epoch,
                                           err, lim)
                             ? 1
                             : 0;
            }
            ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
            if (!ok) break;
            if (SK && n_add > 0) {
                asm volatile("fence.acq_rel.gpu;" ::: "memory");
                io.add = p.partials + (int64_t)((pair + 1) * 2 + (int)rank) * part_floats;
                io.n_add = n_add;
                io.stride = 2 * part_floats;
            }
            tc_fence_after();
            const uint32_t rel = mapa_shared(smem_u32(&acc_empty[ab.s]), 0);
            auto release = [&] {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(rel);
            };
            const int m0 = mt * BT + half * (BT / 2);
            if (m0 < p.M) {
                const uint32_t acc_addr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab.s * BT + half * (BT / 2));
                epilogue_direct<SK>(p, acc_addr, BT / 2, ft * 256 + (int)rank * 128 + q * 32 + lane, m0, release, io,
                                    half * (BT / 2), q * 32 + lane, smem + C::OFF_STG + wi * SS_STG_BOX, lane,
                                    SK || kb0 == 0);
            } else {
                release();  // no token of this half exists
            }
            if (SK && io.write) {
                __threadfence();
                __syncwarp();
                if (lane == 0) flag_publish(p.flags + (pair * 2 + (int)rank) * SS_EPI_WARPS + wi, p.epoch);
            }
            if (SK && n_add > 0) {
                // the warp has read the tail pairs' partials: clear their
                // flags, so that a later launch with the same epoch (a
                // replayed CUDA graph) waits for fresh partials
                __syncwarp();
                if (lane == 0)
                    for (int a = 0; a < n_add; ++a)
                        flag_clear(p.flags + ((pair + 1 + a) * 2 + (int)rank) * SS_EPI_WARPS + wi);
            }
            ab.next<ACC>();
        }
        if (lane == 0) bulk_wait<0>();  // this warp's tensor stores have completed
        __syncwarp();
    }

    tc_fence_before();
    cluster_sync();  // the leader's MMAs and both epilogues are done with both TMEMs
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem, TMEM_COLS);
}

// ---- host launcher --------------------------------------------------------
// Ring depth: as many 64-wide k-block stages as shared memory holds (at most
// 8), rounded down to even so that groups of two k-blocks (one ready wait and
// one commit per group) tile it. Depth pays (the k-loop waits on L2 latency:
// with 256-token tiles, 4 stages measured 13-24 % slower than 6 on the 1.3B
// chunk's linears), but not at the price of single k-block groups (7 stages
// of one k-block measured up to 10 % slower than 6 in groups of two).
constexpr int ss_stages(int bt) {
    const int budget = 227 * 1024 - 1024 - 512 - SS_STG_BYTES;
    const int stage = (bt / 2) * BK * 2 + 128 * BK * 2;
    const int n = budget / stage > 8 ? 8 : budget / stage;
    return n - n % 2;
}

template <int BT, int ACC, int SS, int GRP, bool SK>
static cudaError_t ss_launch_t(const GemmParams &p, int num_sms, cudaStream_t st) {
    using C = SsCfg<BT, ACC, SS>;
    auto kern = gemm_ss_pair_kernel<BT, ACC, SS, GRP, SK>;
    static std::atomic<int> max_pairs_dev[LX2V_MAX_DEVICES];
    std::atomic<int> *slot = device_slot(max_pairs_dev);
    int max_pairs = slot ? slot->load(std::memory_order_relaxed) : 0;
    const int smem = C::SMEM_BYTES;
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof cfg);
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.blockDim = dim3(SS_THREADS);
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
    // stream-K: every pair gets at least one group (the host checked
    // n_tiles * groups >= pairs)
    const long long work = SK ? (long long)n_tiles * (((p.K + BK - 1) / BK) / GRP)
                              : (long long)n_tiles * (p.ksplit > 1 ? p.ksplit : 1);
    const int pairs = work < max_pairs ? (int)work : max_pairs;
    cfg.gridDim = dim3(2 * pairs);
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int BT, int ACC>
static cudaError_t ss_launch_bt(const GemmParams &p, int num_sms, cudaStream_t st) {
    constexpr int SS = ss_stages(BT);
    if constexpr (SS % 2 == 0) {
        if (p.kgroup == 2)
            return p.streamk ? ss_launch_t<BT, ACC, SS, 2, true>(p, num_sms, st)
                             : ss_launch_t<BT, ACC, SS, 2, false>(p, num_sms, st);
    }
    return p.streamk ? ss_launch_t<BT, ACC, SS, 1, true>(p, num_sms, st)
                     : ss_launch_t<BT, ACC, SS, 1, false>(p, num_sms, st);
}

cudaError_t gemm_ss_pair_launch(int bt, const GemmParams &p, int num_sms, cudaStream_t st) {
    switch (bt) {
        case 128: return ss_launch_bt<128, 4>(p, num_sms, st);
        case 192: return ss_launch_bt<192, 2>(p, num_sms, st);
        case 256: return ss_launch_bt<256, 2>(p, num_sms, st);
        default: return cudaErrorInvalidValue;
    }
}

// k-ranges per tile for a reduce-add epilogue (GemmParams::ksplit): the
// fewest that minimise waves x max(k-blocks per item, KSPLIT_MIN_KB) + a fill
// per item. Below ~24 k-blocks an item's k-loop is shorter than a 256 x 256
// tile's epilogue (~8 us), which then no longer hides behind the next item.
// On the 1.3B chunk's FFN2 (114 tiles, 140 k-blocks, 74 pairs) it picks 3:
// 342 items in 5 waves of a third of a tile, against 2 waves of whole tiles.
int gemm_ss_ksplit(int M, int N, int K, int bt, int pairs) {
    constexpr int KSPLIT_MIN_KB = 24, FILL_KB = 2;
    const long long tiles = (long long)((M + bt - 1) / bt) * ((N + 255) / 256);
    const int kb = (K + BK - 1) / BK;
    int best = 1;
    long long best_cost = 0;
    for (int ks = 1; ks <= 4; ++ks) {
        if (kb / ks < 2) break;
        const long long waves = (tiles * ks + pairs - 1) / pairs;
        const long long per = (kb + ks - 1) / ks;
        const long long cost = waves * ((per > KSPLIT_MIN_KB ? per : KSPLIT_MIN_KB) + FILL_KB);
        if (ks == 1 || cost * 20 < best_cost * 19) {  // a new split must win by 5 %
            best = ks;
            best_cost = cost;
        }
    }
    return best;
}

// Token tile for an M x N output on `pairs` CTA pairs. A wave of tiles takes
// time proportional to K * (BT + 150) on B200: a 128-token tile runs its
// k-loop at well under half the time of a 256-token one per wave, since the
// weight tile it streams per k-block is as large (fitted on the 1.3B chunk's
// four linears, M = 4680: it ranks the three tiles as measured for each).
int gemm_ss_token_tile(int M, int N, int K, int pairs) {
    (void)K;
    const int cand[3] = {256, 192, 128};
    int best = 256;
    double best_cost = 0.0;
    for (int i = 0; i < 3; ++i) {
        const int bt = cand[i];
        const long long tiles = (long long)((M + bt - 1) / bt) * ((N + 255) / 256);
        const long long waves = (tiles + pairs - 1) / pairs;
        const double cost = (double)waves * (bt + 150.0);
        if (i == 0 || cost < best_cost) {
            best = bt;
            best_cost = cost;
        }
    }
    return best;
}

}  // namespace lx2v
