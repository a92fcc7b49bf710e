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
//   O  += P_j V_j       tcgen05.mma with A = P_j from TMEM and B = V_j^T from
//                       shared memory (V is given transposed, [D][keys]),
//                       D = O in TMEM
// S is double-buffered, so the softmax of block j overlaps the tensor core's
// S_{j+1} and P_{j-1} V_{j-1}. The running max m only moves when a row's
// new maximum exceeds it by more than 2^8 (then O is rescaled once in TMEM);
// otherwise exp2 arguments stay <= 8 and the final O / l uses the same m, so
// the result is the exact softmax up to rounding.
//
// Masks: none; a bit mask [sq][ceil(sk/32)] (the trait's boolean mask);
// or the DiT's MemRoPE rule tk[key] <= tq[query] with per-block ranges of
// the temporal indices, so that key blocks no query of the tile can see are
// skipped and blocks every query sees are not masked element by element.
// A query that sees no key gets NaN, as the reference's softmax of an
// all -inf row does.
//
// Warp roles (384 threads, one CTA per SM: TMEM 512 columns):
//   warp 0      TMA producer: Q once, then K_j / V_j^T into a 2-stage ring
//   warp 1      TMEM allocator and MMA issuer (one thread)
//   warps 4-11  softmax, then the epilogue (O / l -> out): two warpgroups,
//               each taking half of every S block's key columns (and half of
//               O's columns) for all 128 query rows, so that every scheduler
//               runs two softmax warps
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
constexpr int AT_NS = 2;        // K / V ring stages
constexpr int AT_TILE = 128 * 128 * 2;  // one 128 x 128 bf16 tile: two 64-column SW128 boxes
constexpr int AT_HALF = AT_TILE / 2;
constexpr int AT_OFF_K = AT_TILE;                   // after Q
constexpr int AT_OFF_V = AT_OFF_K + AT_NS * AT_TILE;
constexpr int AT_OFF_BAR = AT_OFF_V + AT_NS * AT_TILE;
// q_full, k_full[NS], k_empty[NS], v_full[NS], v_empty[NS], s_full[2], p_full[2], pv_done, o_full, drain
constexpr int AT_NUM_BARS = 1 + 4 * AT_NS + 2 + 2 + 3;
constexpr int AT_SMEM = 1024 + AT_OFF_BAR + AT_NUM_BARS * 8 + 16 + (512 + 256 + 4) * 4;
constexpr int AT_TMEM_COLS = 512;  // O: 0-127, S/P buffers: 128-255, 256-383
constexpr float AT_RESCALE_LOG2 = 8.0f;

static_assert(AT_SMEM <= 227 * 1024, "shared memory budget");

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Whether key block j can hold a key that some query of the tile sees, and
// whether every query of the tile sees every key of it (no per-element mask).
__device__ __forceinline__ bool block_live(const AttnParams &p, int j, int2 tqr) {
    if (p.mask_mode != ATT_MASK_TEMPORAL) return true;
    return p.tk_range[j].x <= tqr.y;
}
__device__ __forceinline__ bool block_full(const AttnParams &p, int j, int2 tqr) {
    if ((j + 1) * AT_BK > p.sk) return false;
    if (p.mask_mode == ATT_MASK_NONE) return true;
    if (p.mask_mode == ATT_MASK_TEMPORAL) return p.tk_range[j].y <= tqr.x;
    return false;
}

__global__ void __launch_bounds__(384, 1) attention_tc_kernel(const __grid_constant__ AttnParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + AT_OFF_BAR);
    uint64_t *q_full = bars;
    uint64_t *k_full = q_full + 1;
    uint64_t *k_empty = k_full + AT_NS;
    uint64_t *v_full = k_empty + AT_NS;
    uint64_t *v_empty = v_full + AT_NS;
    uint64_t *s_full = v_empty + AT_NS;   // [2]
    uint64_t *p_full = s_full + 2;        // [2]
    uint64_t *pv_done = p_full + 2;
    uint64_t *o_full = pv_done + 1;
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
        for (int s = 0; s < AT_NS; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&s_full[b], 1);
            mbar_init(&p_full[b], 8);
        }
        mbar_init(pv_done, 1);
        mbar_init(o_full, 1);
        mbar_init(drain, 1);
        *reinterpret_cast<volatile int *>(reinterpret_cast<float *>(tmem_slot + 4) + 768) = 0;  // softmax abort flag
        fence_mbar_init();
        tma_prefetch_desc(&p.tmap_q);
        tma_prefetch_desc(&p.tmap_k);
        tma_prefetch_desc(&p.tmap_vt);
    }
    if (warp == 1) tmem_alloc(tmem_slot, AT_TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int last_k[AT_NS], last_v[AT_NS];
            for (int s = 0; s < AT_NS; ++s) last_k[s] = last_v[s] = -1;
            const int qrow = h * p.q_rows + qt * AT_BQ;
            mbar_arrive_expect_tx(q_full, AT_TILE);
            tma_load_2d(smem, &p.tmap_q, q_full, 0, qrow);
            tma_load_2d(smem + AT_HALF, &p.tmap_q, q_full, 64, qrow);
            Ring ks, vs;
            bool ok = true;
            for (int j = 0; j < nblk && ok; ++j) {
                if (!block_live(p, j, tqr)) continue;
                if (!mbar_wait_bounded(&k_empty[ks.s], ks.ph ^ 1, err, lim)) { ok = false; break; }
                uint8_t *kd = smem + AT_OFF_K + ks.s * AT_TILE;
                const int krow = h * p.k_rows + j * AT_BK;
                mbar_arrive_expect_tx(&k_full[ks.s], AT_TILE);
                tma_load_2d(kd, &p.tmap_k, &k_full[ks.s], 0, krow);
                tma_load_2d(kd + AT_HALF, &p.tmap_k, &k_full[ks.s], 64, krow);
                last_k[ks.s] = ks.ph;
                ks.next<AT_NS>();
                if (!mbar_wait_bounded(&v_empty[vs.s], vs.ph ^ 1, err, lim)) { ok = false; break; }
                uint8_t *vd = smem + AT_OFF_V + vs.s * AT_TILE;
                mbar_arrive_expect_tx(&v_full[vs.s], AT_TILE);
                tma_load_2d(vd, &p.tmap_vt, &v_full[vs.s], j * AT_BK, h * AT_D);
                tma_load_2d(vd + AT_HALF, &p.tmap_vt, &v_full[vs.s], j * AT_BK + 64, h * AT_D);
                last_v[vs.s] = vs.ph;
                vs.next<AT_NS>();
            }
            // every issued load lands before the kernel can leave
            mbar_wait_bounded(q_full, 0, nullptr, drain_lim);
            for (int s = 0; s < AT_NS; ++s) {
                if (last_k[s] >= 0) mbar_wait_bounded(&k_full[s], (uint32_t)last_k[s], nullptr, drain_lim);
                if (last_v[s] >= 0) mbar_wait_bounded(&v_full[s], (uint32_t)last_v[s], nullptr, drain_lim);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = idesc_bf16_f32(128, 128);
            const uint32_t q_addr = smem_u32(smem);
            bool ok = mbar_wait_bounded(q_full, 0, err, lim);
            tc_fence_after();
            Ring ks, vs;
            int it = 0;
            auto issue_pv = [&](int i) -> bool {
                if (!mbar_wait_bounded(&p_full[i & 1], (uint32_t)((i >> 1) & 1), err, lim)) return false;
                if (!mbar_wait_bounded(&v_full[vs.s], vs.ph, err, lim)) return false;
                tc_fence_after();
                const uint32_t pbuf = tmem + 128u + (uint32_t)((i & 1) * 128);
                const uint32_t v_addr = smem_u32(smem + AT_OFF_V + vs.s * AT_TILE);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint64_t b = smem_desc_sw128(v_addr + (kk >> 2) * AT_HALF) + (uint64_t)((kk & 3) * 2);
                    mma_ts_f16(tmem, pbuf + (uint32_t)(kk * 8), b, idesc, (i > 0 || kk > 0) ? 1u : 0u);
                }
                mma_commit(&v_empty[vs.s]);
                mma_commit(pv_done);
                vs.next<AT_NS>();
                return true;
            };
            for (int j = 0; j < nblk && ok; ++j) {
                if (!block_live(p, j, tqr)) continue;
                if (!mbar_wait_bounded(&k_full[ks.s], ks.ph, err, lim)) { ok = false; break; }
                tc_fence_after();
                const uint32_t sbuf = tmem + 128u + (uint32_t)((it & 1) * 128);
                const uint32_t k_addr = smem_u32(smem + AT_OFF_K + ks.s * AT_TILE);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint64_t a = smem_desc_sw128(q_addr + (kk >> 2) * AT_HALF) + (uint64_t)((kk & 3) * 2);
                    const uint64_t b = smem_desc_sw128(k_addr + (kk >> 2) * AT_HALF) + (uint64_t)((kk & 3) * 2);
                    mma_ss_f16(sbuf, a, b, idesc, kk > 0 ? 1u : 0u);
                }
                mma_commit(&s_full[it & 1]);
                mma_commit(&k_empty[ks.s]);
                ks.next<AT_NS>();
                if (it >= 1 && !issue_pv(it - 1)) { ok = false; break; }
                ++it;
            }
            if (ok && it >= 1) ok = issue_pv(it - 1);
            if (ok) mma_commit(o_full);
            mma_commit(drain);
            mbar_wait_bounded(drain, 0, nullptr, drain_lim);
        }
        __syncwarp();
    } else if (warp >= 4) {
        // ---------------- softmax + epilogue ----------------
        // Two warpgroups share each query row: warpgroup wg takes the key
        // columns [64 wg, 64 wg + 64) of every S block (and the same half of
        // O's columns). Thread = query row (TMEM lane). The halves' row maxima
        // meet in shared memory, so both warpgroups use the same running max.
        const int wg = (warp - 4) >> 2;
        const int r = (warp & 3) * 32 + lane;
        const int q = qt * AT_BQ + r;
        const bool q_ok = q < p.sq;
        const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        const int tq_row = (p.mask_mode == ATT_MASK_TEMPORAL && q_ok) ? p.tq[q] : 0;
        float *xmax = reinterpret_cast<float *>(tmem_slot + 4);  // [2 blocks][2 warpgroups][128 rows]
        volatile int *abort_flag = reinterpret_cast<volatile int *>(xmax + 768);
        const float NEG_INF = -INFINITY;
        float m_run = NEG_INF, l = 0.0f;
        int it = 0;
        bool ok = true;
        // Both warpgroups meet at a named barrier every block, so neither may
        // leave the loop alone: a failed wait only sets abort_flag, and both
        // leave together right after the next barrier.
        for (int j = 0; j < nblk; ++j) {
            if (!block_live(p, j, tqr)) continue;
            const bool full = block_full(p, j, tqr);
            int okw = 1;
            if (lane == 0) okw = mbar_wait_bounded(&s_full[it & 1], (uint32_t)((it >> 1) & 1), err, lim) ? 1 : 0;
            okw = __shfl_sync(0xFFFFFFFFu, okw, 0);
            if (!okw && lane == 0) *abort_flag = 1;
            tc_fence_after();
            const uint32_t scol = 128u + (uint32_t)((it & 1) * 128);
            // this half's 64 raw scores: two loads in flight, one wait
            uint32_t sv[64];
            if (okw) {
                tmem_ld_32x32b_x32(lane_base + scol + (uint32_t)(wg * 64), *reinterpret_cast<uint32_t(*)[32]>(sv));
                tmem_ld_32x32b_x32(lane_base + scol + (uint32_t)(wg * 64 + 32), *reinterpret_cast<uint32_t(*)[32]>(sv + 32));
                tmem_wait_ld_regs(*reinterpret_cast<uint32_t(*)[32]>(sv));
                tmem_wait_ld_regs(*reinterpret_cast<uint32_t(*)[32]>(sv + 32));
            } else {
#pragma unroll
                for (int i = 0; i < 64; ++i) sv[i] = 0xFF800000u;
            }
            if (!full) {
                // some query of the tile does not see all of this block: the
                // visibility bits of the row's 64 keys (a rolled loop), then
                // -inf where hidden
                const int k0 = j * AT_BK + wg * 64;
                uint32_t vm[2];
#pragma unroll 1
                for (int c = 0; c < 2; ++c) {
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
                for (int i = 0; i < 64; ++i)
                    if (!((vm[i >> 5] >> (i & 31)) & 1u)) sv[i] = 0xFF800000u;  // -inf
            }
            // row max of the raw scores (scale > 0 commutes with max), both halves
            float mx0 = NEG_INF, mx1 = NEG_INF, mx2 = NEG_INF, mx3 = NEG_INF;
#pragma unroll
            for (int i = 0; i < 64; i += 4) {
                mx0 = fmaxf(mx0, __uint_as_float(sv[i]));
                mx1 = fmaxf(mx1, __uint_as_float(sv[i + 1]));
                mx2 = fmaxf(mx2, __uint_as_float(sv[i + 2]));
                mx3 = fmaxf(mx3, __uint_as_float(sv[i + 3]));
            }
            float *xm = xmax + (it & 1) * 256;
            xm[wg * 128 + r] = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
            // also orders both halves' S loads before either half's P stores
            // (P overwrites S's first 64 columns, half of which the other
            // warpgroup reads)
            tc_fence_before();
            named_bar_sync(1, 256);
            tc_fence_after();
            if (*abort_flag) { ok = false; break; }
            const float mx = fmaxf(xm[r], xm[128 + r]) * p.scale_log2;
            const float m_new = fmaxf(m_run, mx);
            const bool need = m_run != NEG_INF && m_new > m_run + AT_RESCALE_LOG2;
            if (__any_sync(0xFFFFFFFFu, need)) {
                // O holds P_0..P_{it-1} V scaled by 2^-m_run: wait for the last
                // of those products, then rescale this warp's rows (this
                // warpgroup's half of the columns) in TMEM
                if (lane == 0) okw = mbar_wait_bounded(pv_done, (uint32_t)((it - 1) & 1), err, lim) ? 1 : 0;
                okw = __shfl_sync(0xFFFFFFFFu, okw, 0);
                if (!okw && lane == 0) *abort_flag = 1;  // both warpgroups leave at the next barrier
                tc_fence_after();
                const float corr = need ? ex2(m_run - m_new) : 1.0f;
#pragma unroll 1
                for (int c = 0; c < 2 && okw; ++c) {
                    const uint32_t oc = (uint32_t)(wg * 64 + c * 32);
                    uint32_t t[32];
                    tmem_ld_32x32b_x32(lane_base + oc, t);
                    tmem_wait_ld_regs(t);
#pragma unroll
                    for (int i = 0; i < 32; ++i) t[i] = __float_as_uint(__uint_as_float(t[i]) * corr);
                    tmem_st_32x32b_x16(lane_base + oc, *reinterpret_cast<uint32_t(*)[16]>(t));
                    tmem_st_32x32b_x16(lane_base + oc + 16u, *reinterpret_cast<uint32_t(*)[16]>(t + 16));
                }
                tmem_wait_st();
                if (need) {
                    l *= corr;
                    m_run = m_new;
                }
            }
            if (m_run == NEG_INF) m_run = m_new;  // nothing visible so far: O holds zeros
            const float nm = m_run == NEG_INF ? 0.0f : -m_run;
            const float sc = p.scale_log2;
            uint32_t pk[32];
            float ls0 = 0.0f, ls1 = 0.0f;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const float a = ex2(fmaf(__uint_as_float(sv[2 * i]), sc, nm));
                const float b = ex2(fmaf(__uint_as_float(sv[2 * i + 1]), sc, nm));
                ls0 += a;
                ls1 += b;
                pk[i] = pack_bf16x2(a, b);
            }
            l += ls0 + ls1;
            // keys [64 wg, 64 wg + 64) -> P columns [32 wg, 32 wg + 32)
            tmem_st_32x32b_x16(lane_base + scol + (uint32_t)(wg * 32), *reinterpret_cast<uint32_t(*)[16]>(pk));
            tmem_st_32x32b_x16(lane_base + scol + (uint32_t)(wg * 32 + 16), *reinterpret_cast<uint32_t(*)[16]>(pk + 16));
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[it & 1]);
            ++it;
        }
        // ---------------- epilogue: out[q, h*D + c] = O / l ----------------
        // every softmax thread arrives here (also after an error) for the row-sum exchange
        float *xl = xmax + 512;
        xl[wg * 128 + r] = l;
        named_bar_sync(1, 256);
        const float lt = xl[r] + xl[128 + r];
        if (ok && it > 0) {
            int okw = 1;
            if (lane == 0) okw = mbar_wait_bounded(o_full, 0, err, lim) ? 1 : 0;
            okw = __shfl_sync(0xFFFFFFFFu, okw, 0);
            ok = okw != 0;
        }
        if (ok) {
            tc_fence_after();
            const float inv = 1.0f / lt;  // lt == 0 (no visible key): NaN, as the reference
            const int64_t obase = (int64_t)q * p.heads * AT_D + (int64_t)h * AT_D + wg * 64;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                uint32_t t[32];
                if (it > 0) {
                    tmem_ld_32x32b_x32(lane_base + (uint32_t)(wg * 64 + c * 32), t);
                    tmem_wait_ld_regs(t);
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) t[i] = 0u;
                }
                if (!q_ok) continue;
                if (p.out_f32) {
                    float4 *dst = reinterpret_cast<float4 *>(reinterpret_cast<float *>(p.out) + obase + c * 32);
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        dst[i] = make_float4(__uint_as_float(t[4 * i]) * inv, __uint_as_float(t[4 * i + 1]) * inv,
                                             __uint_as_float(t[4 * i + 2]) * inv, __uint_as_float(t[4 * i + 3]) * inv);
                } else {
                    uint4 *dst = reinterpret_cast<uint4 *>(reinterpret_cast<__nv_bfloat16 *>(p.out) + obase + c * 32);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        dst[i] = make_uint4(pack_bf16x2(__uint_as_float(t[8 * i]) * inv, __uint_as_float(t[8 * i + 1]) * inv),
                                            pack_bf16x2(__uint_as_float(t[8 * i + 2]) * inv, __uint_as_float(t[8 * i + 3]) * inv),
                                            pack_bf16x2(__uint_as_float(t[8 * i + 4]) * inv, __uint_as_float(t[8 * i + 5]) * inv),
                                            pack_bf16x2(__uint_as_float(t[8 * i + 6]) * inv, __uint_as_float(t[8 * i + 7]) * inv));
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, AT_TMEM_COLS);
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

// ---- V [heads][rows][D] (bf16 or f32) -> V^T [heads][D][sk_pad] bf16, zero past sk ----
__global__ void transpose_v_kernel(const void *v, int v_f32, int heads, int k_rows, int sk, int sk_pad,
                                   __nv_bfloat16 *vt) {
    __shared__ float tile[32][33];
    const int h = blockIdx.z;
    const int k0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int k = k0 + i, c = c0 + threadIdx.x;
        float x = 0.0f;
        if (k < sk) x = ld_act(v, v_f32, ((int64_t)h * k_rows + k) * AT_D + c);
        tile[i][threadIdx.x] = x;
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int c = c0 + i, k = k0 + threadIdx.x;
        if (k < sk_pad) vt[((int64_t)h * AT_D + c) * sk_pad + k] = __float2bfloat16_rn(tile[threadIdx.x][i]);
    }
}

}  // namespace

cudaError_t attention_tc_launch(const AttnParams &p, cudaStream_t st) {
    static std::atomic<int> configured[LX2V_MAX_DEVICES];
    std::atomic<int> *slot = device_slot(configured);
    if (!slot || slot->load() == 0) {
        cudaError_t e = cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AT_SMEM);
        if (e != cudaSuccess) return e;
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

cudaError_t transpose_v_launch(const void *v, int v_f32, int heads, int k_rows, int sk, int sk_pad,
                               __nv_bfloat16 *vt, cudaStream_t st) {
    dim3 grid((sk_pad + 31) / 32, AT_D / 32, heads);
    transpose_v_kernel<<<grid, dim3(32, 8), 0, st>>>(v, v_f32, heads, k_rows, sk, sk_pad, vt);
    return cudaGetLastError();
}

}  // namespace lx2v
