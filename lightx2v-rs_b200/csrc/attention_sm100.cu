// attention_sm100.cu — softmax attention of the DiT on tcgen05 tensor cores.
//
// Computes Backend::attention / Backend::causal_attention
// (crates/lightx2v-core/src/backend.rs:275-307; CPU reference
// crates/lightx2v-cpu/src/lib.rs:171-208):
//   out[q, h*D + c] = sum_k softmax_k(mask(q, k) ? Q[h,q,:].K[h,k,:] / sqrt(D) : -inf) V[h,k,c]
// for q < sq, heads h, D = 128, with bf16 Q/K/V and f32 accumulation.
//
// One CTA per (head, 128-query tile); it walks the key blocks of 128 with an
// online softmax (flash attention):
//   S_j = Q K_j^T       tcgen05.mma kind::f16, A = Q and B = K_j from shared
//                       memory (TMA, 128-byte swizzle), D = S_j in TMEM
//   P_j = exp2(S_j * log2(e)/sqrt(D) - m)   softmax warps, thread = query row:
//                       tcgen05.ld the row, mask, max, exp2, row sum, bf16 P
//                       written back over S_j in TMEM
//   O  += P_j V_j       tcgen05.mma with A = P_j from TMEM and B = V_j from
//                       shared memory as stored ([keys][D]: an MN-major
//                       operand, D contiguous), D = O in TMEM
// The live key blocks alternate between two softmax warpgroups: block i goes
// to warpgroup i % 2, which has its own S buffer, running max m, row sum l and
// accumulator O in TMEM. Each warpgroup's chain (softmax of its block, then
// P V, then the next S into the same buffer) runs while the other
// warpgroup's chain holds the tensor core. P is handed over in two halves of
// 64 keys, so the first half's products run while the softmax computes the
// second. Neither warpgroup waits for the other until the epilogue, which
// merges the two halves:
//   out = (O_0 2^(m_0 - m) + O_1 2^(m_1 - m)) / (l_0 2^(m_0 - m) + l_1 2^(m_1 - m)),
//   m = max(m_0, m_1).
// A running max only moves when a row's new maximum exceeds it by more than
// 2^8 (then that O is rescaled once in TMEM); otherwise exp2 arguments stay
// <= 8, so the result is the exact softmax up to rounding.
//
// Masks: none; a bit mask [sq][ceil(sk/32)] (the trait's boolean mask);
// or the DiT's MemRoPE rule tk[key] <= tq[query] with per-block ranges of
// the temporal indices, so that key blocks no query of the tile can see are
// skipped and blocks every query sees are not masked element by element.
// A query that sees no key gets NaN, as the reference's softmax of an
// all -inf row does.
//
// Warp roles (384 threads, one CTA per SM: TMEM 512 columns):
//   warps 0-7   softmax, then the epilogue (merge, / l -> out): two
//               warpgroups taking alternate key blocks, so that every
//               scheduler runs one softmax warp of each (warp w reads TMEM
//               lanes 32 (w % 4) .. + 31); 208 registers a thread, so that a
//               thread holds a whole 128-key row of S
//   warp 8      TMA producer of Q (once) and K_j (3-stage ring)
//   warp 9      TMEM allocator and MMA issuer (one thread)
//   warp 10     TMA producer of V_j (2-stage ring; keys past sk arrive as zeros)
//   warp 11     idle (warpgroup 2 gives its registers to the softmax)
// Every mbarrier wait is bounded; on expiry the kernel records an error
// word, drains its own copies and MMAs, frees TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <atomic>
#include "attention.h"
#include "gemm_common.cuh"  // Ring, pack_bf16x2, tcgen05 / TMA wrappers, device_slot

namespace lx2v {

namespace {

constexpr int AT_D = 128;       // head_dim of the tensor-core kernel
constexpr int AT_BQ = 128;      // queries per CTA (TMEM lanes)
constexpr int AT_BK = 128;      // keys per block
constexpr int AT_NK = 3;        // K ring stages
constexpr int AT_NV = 2;        // V ring stages
constexpr int AT_TILE = 128 * 128 * 2;  // one 128 x 128 bf16 tile: two 64-column SW128 boxes
constexpr int AT_HALF = AT_TILE / 2;
constexpr int AT_OFF_K = AT_TILE;                   // after Q
constexpr int AT_OFF_V = AT_OFF_K + AT_NK * AT_TILE;
constexpr int AT_OFF_BAR = AT_OFF_V + AT_NV * AT_TILE;
// q_full, k_full[NK], k_empty[NK], v_full[NV], v_empty[NV], s_full[2], p_full[2][2 halves], o_full, drain
constexpr int AT_NUM_BARS = 1 + 2 * AT_NK + 2 * AT_NV + 2 + 4 + 2;
constexpr int AT_SMEM = 1024 + AT_OFF_BAR + AT_NUM_BARS * 8 + 16 + 512 * 4;
constexpr int AT_TMEM_COLS = 512;  // O_0: 0-127, O_1: 128-255, S_0 / P_0: 256-383, S_1 / P_1: 384-511
constexpr float AT_RESCALE_LOG2 = 8.0f;
// registers a block needs after the warpgroups' setmaxnreg: warpgroup 2 (producers,
// MMA issuer) at 72 a thread, the two softmax warpgroups at 208
constexpr int AT_REG_SPLIT = 128 * 72 + 256 * 208;

static_assert(AT_SMEM <= 227 * 1024, "shared memory budget");

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Whether key block j can hold a key that some query of the tile sees
// (bit 0), and whether every query of the tile sees every key of it, so that
// it needs no per-element mask (bit 1).
__device__ __forceinline__ uint32_t block_flags(const AttnParams &p, int j, int2 tqr) {
    const int2 r = p.mask_mode == ATT_MASK_TEMPORAL ? p.tk_range[j] : make_int2(0, 0);
    const bool live = p.mask_mode != ATT_MASK_TEMPORAL || r.x <= tqr.y;
    bool full = (j + 1) * AT_BK <= p.sk;
    if (p.mask_mode == ATT_MASK_TEMPORAL) full = full && r.y <= tqr.x;
    else if (p.mask_mode != ATT_MASK_NONE) full = false;
    return (live ? 1u : 0u) | (full ? 2u : 0u);
}

__global__ void __launch_bounds__(384, 1) attention_tc_kernel(const __grid_constant__ AttnParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + AT_OFF_BAR);
    uint64_t *q_full = bars;
    uint64_t *k_full = q_full + 1;
    uint64_t *k_empty = k_full + AT_NK;
    uint64_t *v_full = k_empty + AT_NK;
    uint64_t *v_empty = v_full + AT_NV;
    uint64_t *s_full = v_empty + AT_NV;   // [2]
    uint64_t *p_full = s_full + 2;        // [2 warpgroups][2 halves]
    uint64_t *o_full = p_full + 4;
    uint64_t *drain = o_full + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // CTAs take the query tiles with the most visible key blocks first (all
    // heads of a tile together), so that the light tiles fill the last wave
    const int h = (int)blockIdx.x % p.heads;
    const int rank_t = (int)blockIdx.x / p.heads;
    const int qt = p.tile_order ? p.tile_order[rank_t] : rank_t;
    const int nblk = (p.sk + AT_BK - 1) / AT_BK;
    const int2 tqr = p.mask_mode == ATT_MASK_TEMPORAL ? p.tq_range[qt] : make_int2(0, 0);
    int *err = p.err;
    const uint64_t lim = p.wait_limit_ns;
    const uint64_t drain_lim = lim > 500000000ull ? lim : 500000000ull;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < AT_NK; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
        }
        for (int s = 0; s < AT_NV; ++s) {
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&s_full[b], 1);
            mbar_init(&p_full[2 * b], 4);
            mbar_init(&p_full[2 * b + 1], 4);
        }
        mbar_init(o_full, 1);
        mbar_init(drain, 1);
        fence_mbar_init();
        tma_prefetch_desc(&p.tmap_q);
        tma_prefetch_desc(&p.tmap_k);
        tma_prefetch_desc(&p.tmap_v);
    }
    if (warp == 9) tmem_alloc(tmem_slot, AT_TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp >= 8) {
    // Registers: the kernel is launched with 168 a thread (384 x 168 =
    // 64512). Warpgroup 2 (producer, MMA issuer, two idle warps) gives back
    // down to 72 and the softmax warpgroups take 208, which holds a whole
    // 128-key row of S: 128 x 72 + 256 x 208 = 62464 <= 64512.
    asm volatile("setmaxnreg.dec.sync.aligned.u32 72;" ::: "memory");
    if (warp == 8 || warp == 10) {
        // ---------------- TMA producers: warp 8 Q and K_j, warp 10 V_j ----------------
        // (separate threads, so that a K load never waits behind the
        // release of a V stage, which comes only after that block's softmax)
        if (lane == 0) {
            const bool is_k = warp == 8;
            uint64_t *full = is_k ? k_full : v_full;
            uint64_t *empty = is_k ? k_empty : v_empty;
            const int ns = is_k ? AT_NK : AT_NV;
            int last[AT_NK];
            for (int s = 0; s < AT_NK; ++s) last[s] = -1;
            if (is_k) {
                const int qrow = h * p.q_rows + qt * AT_BQ;
                mbar_arrive_expect_tx(q_full, AT_TILE);
                tma_load_2d(smem, &p.tmap_q, q_full, 0, qrow);
                tma_load_2d(smem + AT_HALF, &p.tmap_q, q_full, 64, qrow);
            }
            int st = 0;
            uint32_t ph = 0;
            for (int j = 0; j < nblk; ++j) {
                if (!(block_flags(p, j, tqr) & 1u)) continue;
                if (!mbar_wait_bounded(&empty[st], ph ^ 1, err, lim)) break;
                mbar_arrive_expect_tx(&full[st], AT_TILE);
                if (is_k) {
                    uint8_t *kd = smem + AT_OFF_K + st * AT_TILE;
                    const int krow = h * p.k_rows + j * AT_BK;
                    tma_load_2d(kd, &p.tmap_k, &full[st], 0, krow);
                    tma_load_2d(kd + AT_HALF, &p.tmap_k, &full[st], 64, krow);
                } else {
                    uint8_t *vd = smem + AT_OFF_V + st * AT_TILE;
                    tma_load_3d(vd, &p.tmap_v, &full[st], 0, j * AT_BK, h);
                    tma_load_3d(vd + AT_HALF, &p.tmap_v, &full[st], 64, j * AT_BK, h);
                }
                last[st] = (int)ph;
                if (++st == ns) {
                    st = 0;
                    ph ^= 1u;
                }
            }
            // every issued load lands before the kernel can leave
            if (is_k) mbar_wait_bounded(q_full, 0, nullptr, drain_lim);
            for (int s = 0; s < ns; ++s)
                if (last[s] >= 0) mbar_wait_bounded(&full[s], (uint32_t)last[s], nullptr, drain_lim);
        }
        __syncwarp();
    } else if (warp == 9) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = idesc_bf16_f32(128, 128);
            // P V reads B = V_j as stored: MN-major (bit 16 of the instruction
            // descriptor), 128-byte swizzle; each 64-column half of D is one
            // TMA box of 128 keys x 128 B (LBO: the 16 KB between the halves),
            // 8 keys per 1 KB swizzle atom (SBO), 16 keys (2 KB) per MMA
            const uint32_t idesc_pv = idesc | (1u << 16);
            const uint32_t q_addr = smem_u32(smem);
            bool ok = mbar_wait_bounded(q_full, 0, err, lim);
            tc_fence_after();
            Ring ks, vs;
            int it = 0;
            // block i (counted over live blocks) belongs to softmax warpgroup
            // i % 2: S_i goes to its S buffer, P_i V_i into its accumulator
            auto issue_pv = [&](int i) -> bool {
                const int wg = i & 1;
                if (!mbar_wait_bounded(&v_full[vs.s], vs.ph, err, lim)) return false;
                const uint32_t pbuf = tmem + 256u + (uint32_t)(wg * 128);
                const uint32_t obuf = tmem + (uint32_t)(wg * 128);
                const uint32_t v_addr = smem_u32(smem + AT_OFF_V + vs.s * AT_TILE);
                // P arrives in two halves of 64 keys: the first half's
                // products start while the softmax still computes the second
                for (int hf = 0; hf < 2; ++hf) {
                    if (!mbar_wait_bounded(&p_full[2 * wg + hf], (uint32_t)((i >> 1) & 1), err, lim)) return false;
                    tc_fence_after();
#pragma unroll
                    for (int k4 = 0; k4 < 4; ++k4) {
                        const int kk = 4 * hf + k4;
                        const uint64_t b = smem_desc_sw128_mn(v_addr + (uint32_t)(kk * 2048), AT_HALF);
                        mma_ts_f16(obuf, pbuf + (uint32_t)(kk * 8), b, idesc_pv, (i >= 2 || kk > 0) ? 1u : 0u);
                    }
                }
                mma_commit(&v_empty[vs.s]);
                vs.next<AT_NV>();
                return true;
            };
            for (int j = 0; j < nblk && ok; ++j) {
                if (!(block_flags(p, j, tqr) & 1u)) continue;
                if (!mbar_wait_bounded(&k_full[ks.s], ks.ph, err, lim)) { ok = false; break; }
                tc_fence_after();
                const uint32_t sbuf = tmem + 256u + (uint32_t)((it & 1) * 128);
                const uint32_t k_addr = smem_u32(smem + AT_OFF_K + ks.s * AT_TILE);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint64_t a = smem_desc_sw128(q_addr + (kk >> 2) * AT_HALF) + (uint64_t)((kk & 3) * 2);
                    const uint64_t b = smem_desc_sw128(k_addr + (kk >> 2) * AT_HALF) + (uint64_t)((kk & 3) * 2);
                    mma_ss_f16(sbuf, a, b, idesc, kk > 0 ? 1u : 0u);
                }
                mma_commit(&s_full[it & 1]);
                mma_commit(&k_empty[ks.s]);
                ks.next<AT_NK>();
                if (it >= 1 && !issue_pv(it - 1)) { ok = false; break; }
                ++it;
            }
            if (ok && it >= 1) ok = issue_pv(it - 1);
            if (ok) mma_commit(o_full);
            mma_commit(drain);
            mbar_wait_bounded(drain, 0, nullptr, drain_lim);
        }
        __syncwarp();
    }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 208;" ::: "memory");
        // ---------------- softmax + epilogue ----------------
        // Warpgroup wg takes the live key blocks of parity wg (block number
        // it, counted over live blocks, with it % 2 == wg): whole 128-key rows
        // of S_wg, its own running max m and row sum l, and its own
        // accumulator O_wg. The two warpgroups never wait for each other
        // inside the loop, so one's TMEM loads and max overlap the other's
        // exponentials. Thread = query row (TMEM lane).
        const int wg = warp >> 2;
        const int r = (warp & 3) * 32 + lane;
        const int q = qt * AT_BQ + r;
        const bool q_ok = q < p.sq;
        const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        const uint32_t o_col = (uint32_t)(wg * 128);
        const uint32_t s_col = 256u + (uint32_t)(wg * 128);
        const int tq_row = (p.mask_mode == ATT_MASK_TEMPORAL && q_ok) ? p.tq[q] : 0;
        const float NEG_INF = -INFINITY;
        const float sc = p.scale_log2;
        float m_run = NEG_INF, l = 0.0f;
        int it = 0, n_mine = 0;
        bool ok = true;
        for (int j = 0; j < nblk; ++j) {
            const uint32_t bf = block_flags(p, j, tqr);
            if (!(bf & 1u)) continue;
            const bool mine = (it & 1) == wg;
            ++it;
            if (!mine) continue;
            const int i = n_mine++;
            const bool full = (bf & 2u) != 0;
            int okw = 1;
            if (lane == 0) okw = mbar_wait_bounded(&s_full[wg], (uint32_t)(i & 1), err, lim) ? 1 : 0;
            okw = __shfl_sync(0xFFFFFFFFu, okw, 0);
            if (!okw) { ok = false; break; }  // warp-uniform; the waits of the others end on the error word
            tc_fence_after();
            // the block's 128 raw scores: four loads in flight, then the waits
            uint32_t sv[128];
#pragma unroll
            for (int c = 0; c < 4; ++c)
                tmem_ld_32x32b_x32(lane_base + s_col + (uint32_t)(c * 32), *reinterpret_cast<uint32_t(*)[32]>(sv + 32 * c));
#pragma unroll
            for (int c = 0; c < 4; ++c) tmem_wait_ld_regs(*reinterpret_cast<uint32_t(*)[32]>(sv + 32 * c));
            if (!full) {
                // some query of the tile does not see all of this block: the
                // visibility bits of the row's 128 keys (a rolled loop), then
                // -inf where hidden
                const int k0 = j * AT_BK;
                uint32_t vm[4];
#pragma unroll 1
                for (int c = 0; c < 4; ++c) {
                    uint32_t w = 0;
                    const int kc = k0 + c * 32;
                    if (p.mask_mode == ATT_MASK_BITS && q_ok && kc < p.sk) {
                        w = __ldg(p.mask_bits + h * p.mask_head_stride + (int64_t)q * p.mask_words + (kc >> 5));
                    } else if (p.mask_mode == ATT_MASK_TEMPORAL && q_ok) {
#pragma unroll 1
                        for (int b = 0; b < 32; ++b)
                            if (kc + b < p.sk && __ldg(p.tk + kc + b) <= tq_row) w |= 1u << b;
                    } else {
                        w = 0xFFFFFFFFu;
                    }
                    const int valid = p.sk - kc;  // keys past sk are never visible
                    if (valid < 32) w &= valid <= 0 ? 0u : ((1u << valid) - 1u);
                    vm[c] = w;
                }
#pragma unroll
                for (int k = 0; k < 128; ++k)
                    if (!((vm[k >> 5] >> (k & 31)) & 1u)) sv[k] = 0xFF800000u;  // -inf
            }
            // row max of the raw scores (scale > 0 commutes with max)
            float mx0 = NEG_INF, mx1 = NEG_INF, mx2 = NEG_INF, mx3 = NEG_INF;
#pragma unroll
            for (int k = 0; k < 128; k += 4) {
                mx0 = fmaxf(mx0, __uint_as_float(sv[k]));
                mx1 = fmaxf(mx1, __uint_as_float(sv[k + 1]));
                mx2 = fmaxf(mx2, __uint_as_float(sv[k + 2]));
                mx3 = fmaxf(mx3, __uint_as_float(sv[k + 3]));
            }
            const float mx = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * sc;
            const float m_new = fmaxf(m_run, mx);
            const bool need = m_run != NEG_INF && m_new > m_run + AT_RESCALE_LOG2;
            if (__any_sync(0xFFFFFFFFu, need)) {
                // O_wg holds this warpgroup's earlier P V products scaled by
                // 2^-m_run. The last of them (block i-1 of this warpgroup) was
                // issued before the product that filled S_wg, so the S_wg
                // wait above has already seen it complete: rescale this
                // warp's rows of O_wg in TMEM.
                const float corr = need ? ex2(m_run - m_new) : 1.0f;
#pragma unroll 1
                for (int c = 0; c < 4; ++c) {
                    const uint32_t oc = o_col + (uint32_t)(c * 32);
                    uint32_t t[32];
                    tmem_ld_32x32b_x32(lane_base + oc, t);
                    tmem_wait_ld_regs(t);
#pragma unroll
                    for (int k = 0; k < 32; ++k) t[k] = __float_as_uint(__uint_as_float(t[k]) * corr);
                    tmem_st_32x32b_x16(lane_base + oc, *reinterpret_cast<uint32_t(*)[16]>(t));
                    tmem_st_32x32b_x16(lane_base + oc + 16u, *reinterpret_cast<uint32_t(*)[16]>(t + 16));
                }
                if (need) {
                    l *= corr;
                    m_run = m_new;
                }
            }
            if (m_run == NEG_INF) m_run = m_new;  // nothing visible so far: O_wg holds zeros
            const float nm = m_run == NEG_INF ? 0.0f : -m_run;
            // P = exp2(S * scale - m) as bf16 pairs over the first 64 columns
            // of S_wg (all 128 scores are already in registers)
            // the exponent arguments and the row sums two at a time (f32x2:
            // one packed FMA / add for a pair of keys, the same rounding and
            // the same two partial sums as the scalar form)
            uint64_t ls2, sc2, nm2;
            asm("mov.b64 %0, {%1, %1};" : "=l"(sc2) : "f"(sc));
            asm("mov.b64 %0, {%1, %1};" : "=l"(nm2) : "f"(nm));
            asm("mov.b64 %0, {%1, %1};" : "=l"(ls2) : "f"(0.0f));
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                uint32_t pk[16];
#pragma unroll
                for (int k = 0; k < 16; ++k) {
                    uint64_t s2, x2, p2;
                    float xa, xb;
                    asm("mov.b64 %0, {%1, %2};" : "=l"(s2) : "r"(sv[32 * c + 2 * k]), "r"(sv[32 * c + 2 * k + 1]));
                    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(x2) : "l"(s2), "l"(sc2), "l"(nm2));
                    asm("mov.b64 {%0, %1}, %2;" : "=f"(xa), "=f"(xb) : "l"(x2));
                    const float a = ex2(xa);
                    const float b = ex2(xb);
                    asm("mov.b64 %0, {%1, %2};" : "=l"(p2) : "f"(a), "f"(b));
                    asm("add.rn.f32x2 %0, %0, %1;" : "+l"(ls2) : "l"(p2));
                    pk[k] = pack_bf16x2(a, b);
                }
                tmem_st_32x32b_x16(lane_base + s_col + (uint32_t)(c * 16), pk);
                if (c == 1 || c == 3) {  // keys [0, 64) and [64, 128) of P are in TMEM
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&p_full[2 * wg + (c >> 1)]);
                }
            }
            float ls0, ls1;
            asm("mov.b64 {%0, %1}, %2;" : "=f"(ls0), "=f"(ls1) : "l"(ls2));
            l += ls0 + ls1;
        }
        // ---------------- epilogue: out[q, h*D + c] = (O_0 a_0 + O_1 a_1) / (l_0 a_0 + l_1 a_1) ----------------
        // with a_w = 2^(m_w - max(m_0, m_1)); every softmax thread arrives
        // here (also after an error) for the exchange of m and l
        float *xm = reinterpret_cast<float *>(tmem_slot + 4);  // [2 warpgroups][128 rows] m, then l
        xm[wg * 128 + r] = m_run;
        xm[256 + wg * 128 + r] = l;
        named_bar_sync(1, 256);
        const float m0 = xm[r], m1 = xm[128 + r];
        const float mt = fmaxf(m0, m1);
        // a warpgroup that saw nothing of this row (or had no block at all:
        // O_w never written) contributes nothing
        const float a0 = m0 == NEG_INF ? 0.0f : ex2(m0 - mt);
        const float a1 = m1 == NEG_INF ? 0.0f : ex2(m1 - mt);
        const float lt = xm[256 + r] * a0 + xm[384 + r] * a1;
        if (ok && it > 0) {
            int okw = 1;
            if (lane == 0) okw = mbar_wait_bounded(o_full, 0, err, lim) ? 1 : 0;
            okw = __shfl_sync(0xFFFFFFFFu, okw, 0);
            ok = okw != 0;
        }
        if (ok) {
            tc_fence_after();
            const float inv = 1.0f / lt;  // lt == 0 (no visible key): NaN, as the reference
            // this warpgroup writes output columns [64 wg, 64 wg + 64)
            const int64_t obase = (int64_t)q * p.heads * AT_D + (int64_t)h * AT_D + wg * 64;
#pragma unroll 1
            for (int c = 0; c < 2; ++c) {
                const uint32_t oc = (uint32_t)(wg * 64 + c * 32);
                uint32_t t0[32], t1[32];
                tmem_ld_32x32b_x32(lane_base + oc, t0);
                tmem_ld_32x32b_x32(lane_base + 128u + oc, t1);
                tmem_wait_ld_regs(t0);
                tmem_wait_ld_regs(t1);
                float o[32];
#pragma unroll
                for (int k = 0; k < 32; ++k) {
                    const float v0 = a0 != 0.0f ? __uint_as_float(t0[k]) * a0 : 0.0f;
                    const float v1 = a1 != 0.0f ? __uint_as_float(t1[k]) * a1 : 0.0f;
                    o[k] = (v0 + v1) * inv;
                }
                if (!q_ok) continue;
                if (p.out_f32) {
                    float4 *dst = reinterpret_cast<float4 *>(reinterpret_cast<float *>(p.out) + obase + c * 32);
#pragma unroll
                    for (int k = 0; k < 8; ++k) dst[k] = make_float4(o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]);
                } else {
                    uint4 *dst = reinterpret_cast<uint4 *>(reinterpret_cast<__nv_bfloat16 *>(p.out) + obase + c * 32);
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        dst[k] = make_uint4(pack_bf16x2(o[8 * k], o[8 * k + 1]), pack_bf16x2(o[8 * k + 2], o[8 * k + 3]),
                                            pack_bf16x2(o[8 * k + 4], o[8 * k + 5]), pack_bf16x2(o[8 * k + 6], o[8 * k + 7]));
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 9) tmem_dealloc(tmem, AT_TMEM_COLS);
}

// ---- generic kernel (any head_dim <= 256, f32 or bf16 buffers) ----------------
// One CTA per (head, query): scores of all keys in shared memory (the same
// sequential-d dot products and scale as the reference), a block max, exp,
// block sum, then out[c] = sum_k p_k v[k][c] accumulated over k in order by
// thread c. A GPU kernel for the shapes the tensor-core kernel does not take
// (head_dim != 128, f32 operands); not a fast path.
__device__ __forceinline__ float ld_act(const void *p, int f32, int64_t i) {
    return f32 ? reinterpret_cast<const float *>(p)[i] : __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[i]);
}

__global__ void __launch_bounds__(128) attention_simt_kernel(AttnSimtParams p) {
    extern __shared__ float sc[];  // [sk] scores, then [32] reduction scratch
    float *red = sc + p.sk;
    const int h = (int)blockIdx.x / p.sq, q = (int)blockIdx.x % p.sq;
    const int D = p.d;
    const float scale = 1.0f / sqrtf((float)D);
    const int64_t qbase = ((int64_t)h * p.q_rows + q) * D;
    float lmax = -INFINITY;
    for (int k = threadIdx.x; k < p.sk; k += blockDim.x) {
        bool vis = true;
        if (p.mask_mode == ATT_MASK_TEMPORAL) vis = p.tk[k] <= p.tq[q];
        else if (p.mask_mode == ATT_MASK_BITS)
            vis = (p.mask_bits[h * p.mask_head_stride + (int64_t)q * p.mask_words + (k >> 5)] >> (k & 31)) & 1u;
        float s = -INFINITY;
        if (vis) {
            const int64_t kbase = ((int64_t)h * p.k_rows + k) * D;
            float acc = 0.0f;
            for (int c = 0; c < D; ++c) acc = fmaf(ld_act(p.q, p.qkv_f32, qbase + c), ld_act(p.k, p.qkv_f32, kbase + c), acc);
            s = acc * scale;
        }
        sc[k] = s;
        lmax = fmaxf(lmax, s);
    }
    for (int o = 16; o > 0; o >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xFFFFFFFFu, lmax, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = lmax;
    __syncthreads();
    float m = -INFINITY;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, red[w]);
    __syncthreads();
    float lsum = 0.0f;
    for (int k = threadIdx.x; k < p.sk; k += blockDim.x) {
        const float e = expf(sc[k] - m);
        sc[k] = e;
        lsum += e;
    }
    for (int o = 16; o > 0; o >>= 1) lsum += __shfl_xor_sync(0xFFFFFFFFu, lsum, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = lsum;
    __syncthreads();
    float sum = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) sum += red[w];
    const float inv = 1.0f / sum;
    for (int c = threadIdx.x; c < D; c += blockDim.x) {
        float acc = 0.0f;
        for (int k = 0; k < p.sk; ++k) acc = fmaf(sc[k] * inv, ld_act(p.v, p.qkv_f32, ((int64_t)h * p.k_rows + k) * D + c), acc);
        const int64_t oi = (int64_t)q * p.heads * D + (int64_t)h * D + c;
        if (p.out_f32) reinterpret_cast<float *>(p.out)[oi] = acc;
        else reinterpret_cast<__nv_bfloat16 *>(p.out)[oi] = __float2bfloat16_rn(acc);
    }
}

}  // namespace

cudaError_t attention_tc_launch(const AttnParams &p, cudaStream_t st) {
    static std::atomic<int> configured[LX2V_MAX_DEVICES];
    std::atomic<int> *slot = device_slot(configured);
    if (!slot || slot->load() == 0) {
        cudaError_t e = cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AT_SMEM);
        if (e != cudaSuccess) return e;
        // the warpgroups' register split (setmaxnreg: 128 x 72 + 256 x 208)
        // must fit in what the block is launched with, or the increase
        // would wait forever: refuse to launch a build that has fewer
        cudaFuncAttributes fa;
        e = cudaFuncGetAttributes(&fa, attention_tc_kernel);
        if (e != cudaSuccess) return e;
        if (fa.numRegs * 384 < AT_REG_SPLIT) return cudaErrorInvalidConfiguration;
        if (slot) slot->store(1);
    }
    const int n_qt = (p.sq + AT_BQ - 1) / AT_BQ;
    attention_tc_kernel<<<n_qt * p.heads, 384, AT_SMEM, st>>>(p);
    return cudaGetLastError();
}

cudaError_t attention_simt_launch(const AttnSimtParams &p, cudaStream_t st) {
    const size_t smem = ((size_t)p.sk + 32) * sizeof(float);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(attention_simt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
    }
    attention_simt_kernel<<<p.heads * p.sq, 128, smem, st>>>(p);
    return cudaGetLastError();
}


}  // namespace lx2v
