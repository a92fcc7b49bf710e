// gemm_common.cuh — pieces shared by the single-CTA and the CTA-pair
// tensor-core linear kernels: stage layout of the weight codes, the per-item
// decode (smem codes -> bf16 pairs for tcgen05.st), the GELU epilogue math and
// the epilogue tile writer (TMEM -> registers -> smem staging -> coalesced
// global stores or vector reductions).
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include "dequant.cuh"
#include "gemm.h"
#include "ptx.cuh"

namespace lx2v {

constexpr int BK = 64;          // k columns per pipeline stage
// Epilogue staging: one [32 tokens][32 features] f32 tile per epilogue warp,
// rows padded to 36 floats (column writes and 16-byte row reads both run at
// the minimum number of shared-memory wavefronts).
constexpr int STG_PITCH = 36;
constexpr int STG_WARP_FLOATS = 32 * STG_PITCH;
constexpr int STG_TOTAL = 4 * STG_WARP_FLOATS * 4;  // bytes, four epilogue warps
constexpr int EPI_THREADS = 128;
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

// A ring position (stage, phase), advanced per item without divisions.
struct Ring {
    int s = 0, ph = 0;
    template <int N>
    __device__ __forceinline__ void next() {
        if (++s == N) { s = 0; ph ^= 1; }
    }
};

__device__ __forceinline__ uint2 lds64(const uint8_t *p) {
    return *reinterpret_cast<const uint2 *>(p);
}

// Decode UNITS consecutive 16-value units of weight row `r` of one stage,
// starting at unit `u0` (columns 16*u0 ..) of k-block `kb`, from the stage's
// code tile `wstage`, scale words `sstage` and FP8 flags `fstage` in shared
// memory. Output: 8 bf16x2 words per unit, columns (2i, 2i+1) -> word i.
// Scale-group index of a unit inside the stage's scale box: the box starts
// at the k-block's first group; groups are >= 16 columns and either divide
// 64 (p.gshift = log2(group)) or are multiples of 64 (p.gshift = 6).
// FP8: every unit first takes the branch-free hardware-converter path; only
// when some row of the warp has a flagged block (special codes or an extreme
// scale, rare) are those rows' units decoded again on the exact slow path.
// Keeping the common path free of per-unit branches lets the compiler overlap
// the units' shared-memory loads.
template <int FMT, int UNITS>
__device__ __forceinline__ void decode_units(const GemmParams &p, const uint8_t *wstage, const uint8_t *sstage,
                                             const uint8_t *fstage, int r, int u0, uint32_t (&packed)[8 * UNITS]) {
    const uint8_t *wt = wstage + r * WTile<FMT>::ROW_BYTES;
#pragma unroll
    for (int u = 0; u < UNITS; ++u) {
        const int ui = u0 + u;
        uint32_t *out = packed + 8 * u;
        uint32_t o[8];
        if (FMT == FMT_BF16) {
            // 128-byte rows, 128B swizzle: 16-byte chunk ^= row & 7; a unit is 2 chunks
            const uint4 a = lds128(wt + (((2 * ui) ^ (r & 7)) << 4));
            const uint4 b = lds128(wt + (((2 * ui + 1) ^ (r & 7)) << 4));
            o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
            o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
        } else {
            const uint32_t *sw = reinterpret_cast<const uint32_t *>(sstage);
            const int gi = (ui * 16) >> p.gshift;
            if (FMT == FMT_Q4) {
                // 32-byte rows, 32B swizzle: chunk ^= (row >> 2) & 1; a unit is half a chunk
                const uint2 raw = lds64(wt + (((ui >> 1) ^ ((r >> 2) & 1)) << 4) + (ui & 1) * 8);
                float s, z;
                q4_scale_zero(sw[gi * 128 + r], s, z);
                unit_to_bf16<FMT_Q4>(make_uint4(raw.x, raw.y, 0, 0), make_uint4(0, 0, 0, 0), s, z, 0, o);
            } else {
                // 64-byte rows, 64B swizzle: chunk ^= (row >> 1) & 3; a unit is one chunk
                const uint4 raw = lds128(wt + ((ui ^ ((r >> 1) & 3)) << 4));
                const float s = __uint_as_float(sw[r]);
                unit_to_bf16<FMT>(raw, raw, s, 0.0f, 0, o);
            }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) out[i] = o[i];
    }
    if (FMT == FMT_FP8) {
        int flagged = 0;
#pragma unroll
        for (int u = 0; u < UNITS; u += 2) flagged |= fstage[((u0 + u) >> 1) * 128 + r];
        if (__any_sync(0xFFFFFFFFu, flagged != 0) && flagged != 0) {
            const uint32_t *sw = reinterpret_cast<const uint32_t *>(sstage);
#pragma unroll
            for (int u = 0; u < UNITS; ++u) {
                const int ui = u0 + u;
                const int mode = fstage[(ui >> 1) * 128 + r];
                if (mode != 0) {
                    const uint4 raw = lds128(wt + ((ui ^ ((r >> 1) & 3)) << 4));
                    const PackedUnit pu = fp8_unit_special(raw, __uint_as_float(sw[r]), mode);
#pragma unroll
                    for (int i = 0; i < 8; ++i) packed[8 * u + i] = pu.w[i];
                }
            }
        }
    }
}

// The work of one CTA pair as a list of segments: k-blocks [kb0, kb1) of a
// tile. Whole tiles: tiles pair, pair + npairs, ... Stream-K: the first `dp`
// tiles as whole tiles in that order (dp is a multiple of npairs: full waves,
// so the pairs running at the same time keep sharing operand tiles in L2),
// then the remaining tiles' k-blocks split into npairs equal contiguous
// ranges [lo, hi) (counted from tile 0); a range may start and end inside a
// tile. dp = 0 splits everything.
struct PairWork {
    long long lo = 0, hi = 0;  // stream-K k-block range
    int KB = 1, pair = 0, npairs = 1, my_tiles = 0;
    // whole-tile mode: ks k-ranges per tile, items range-major (item u is
    // range u / n_tiles of tile u % n_tiles), so the pairs running at the
    // same time share k-ranges of x; my_tiles counts this pair's items
    int ks = 1, n_tiles = 0;
    int dp = 0, my_dp = 0;     // whole tiles before the split range (all pairs / this pair)
    bool sk = false;
    __host__ __device__ __forceinline__ void init_split(int n_tiles, int dp_tiles) {
        // The split range must give every pair at least one k-block: a pair
        // with an empty range would be counted by the head of a tile it has
        // no part of. When the leftover tiles are too few, split one more
        // wave as well (dp stays a multiple of npairs).
        if (dp_tiles >= npairs && (long long)(n_tiles - dp_tiles) * KB < npairs) dp_tiles -= npairs;
        dp = dp_tiles;
        my_dp = pair < dp ? (dp - 1 - pair) / npairs + 1 : 0;
        const long long rem = (long long)(n_tiles - dp) * KB;
        lo = (long long)dp * KB + rem * pair / npairs;
        hi = (long long)dp * KB + rem * (pair + 1) / npairs;
    }
    // first k-block (counted from tile 0) of pair q's split range
    __host__ __device__ __forceinline__ long long split_start(int n_tiles, int q) const {
        return (long long)dp * KB + (long long)(n_tiles - dp) * KB * q / npairs;
    }
    __host__ __device__ __forceinline__ int count() const {
        if (!sk) return my_tiles;
        return my_dp + (hi > lo ? (int)((hi - 1) / KB - lo / KB + 1) : 0);
    }
    __host__ __device__ __forceinline__ long long total_kb() const {
        return sk ? (long long)my_dp * KB + (hi - lo) : (long long)my_tiles * KB;
    }
    __host__ __device__ __forceinline__ void seg(int idx, int &tile, int &kb0, int &kb1) const {
        if (!sk || idx < my_dp) {
            tile = pair + idx * npairs;
            kb0 = 0;
            kb1 = KB;
            if (!sk && ks > 1) {
                const int part = tile / n_tiles;
                tile -= part * n_tiles;
                kb0 = (int)((long long)part * KB / ks);
                kb1 = (int)((long long)(part + 1) * KB / ks);
            }
            return;
        }
        const long long t = lo / KB + (idx - my_dp);
        const long long start = lo > t * KB ? lo : t * KB;
        const long long end = hi < (t + 1) * KB ? hi : (t + 1) * KB;
        tile = (int)t;
        kb0 = (int)(start - t * KB);
        kb1 = (int)(end - t * KB);
    }
};

// Partial-tile traffic of a stream-K epilogue (see GemmParams::streamk).
struct PartialIO {
    float *write = nullptr;        // non-null: store the raw accumulator here, nothing else
    const float *add = nullptr;    // non-null: add n_add partial tiles from here before the epilogue
    int n_add = 0;
    int64_t add_stride = 0;        // floats between consecutive partial tiles
};

// Epilogue of one accumulator tile held in this CTA's TMEM: 128 features
// (lanes; this thread = feature f_base + 32*q + lane) x `ntok` tokens
// (columns from `acc_addr`, tokens m0 .. m0 + ntok). Bias, GELU and gate are
// applied in f32. Each warp transposes its 32 features x 32 tokens through
// its own staging tile and then writes, per thread, one token's 32 features
// (64 or 128 contiguous bytes of y) with 16-byte stores, or vector reductions
// into h for the gated residual; warps never wait for each other. `release`
// runs once the last TMEM load of the tile has completed (the accumulator can
// be reused from then on). Partial tiles (`io`) are stored token-major,
// [token][128 features] f32, so a warp's accesses for one token are 128
// contiguous bytes.
template <bool PARTIAL = false, typename Release>
__device__ __forceinline__ void epilogue_tile(const GemmParams &p, uint32_t acc_addr, int ntok, int f_base,
                                              int m0, int q, int lane, uint8_t *stg_base, Release release,
                                              const PartialIO &io = PartialIO()) {
    const int et = q * 32 + lane;  // 0..127
    const int f = f_base + et;
    float bias_f = 0.0f, gate_f = 1.0f;
    if (f < p.N) {
        if (p.bias) bias_f = p.bias_f32 ? reinterpret_cast<const float *>(p.bias)[f]
                                        : __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p.bias)[f]);
        if (p.gate) gate_f = p.gate_f32 ? reinterpret_cast<const float *>(p.gate)[f]
                                        : __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p.gate)[f]);
    }
    const float2 bias2 = make_float2(bias_f, bias_f), gate2 = make_float2(gate_f, gate_f);
    float *stg = reinterpret_cast<float *>(stg_base) + q * STG_WARP_FLOATS;
    const int fw = f_base + 32 * q;  // first feature of this warp
    const int nvalid = p.N - fw;     // this warp's features inside N (N % 16 == 0)
    const int nld = min(ntok / 32, (p.M - m0 + 31) / 32);
    for (int c = 0; c < nld; ++c) {
        uint32_t acc[32];
        tmem_ld_32x32b_x32(acc_addr + (uint32_t)(c * 32), acc);
        tmem_wait_ld();
        if (c == nld - 1) release();
        if (PARTIAL) {
            if (io.write) {
                float *dst = io.write + (int64_t)(c * 32) * 128 + et;
#pragma unroll
                for (int i = 0; i < 32; ++i) __stcg(dst + i * 128, __uint_as_float(acc[i]));
                continue;
            }
            for (int part = 0; part < io.n_add; ++part) {
                const float *src = io.add + part * io.add_stride + (int64_t)(c * 32) * 128 + et;
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    acc[i] = __float_as_uint(__uint_as_float(acc[i]) + __ldcg(src + i * 128));
            }
        }
        __syncwarp();  // the previous chunk's rows have been read
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            float2 t = __fadd2_rn(make_float2(__uint_as_float(acc[2 * i]), __uint_as_float(acc[2 * i + 1])), bias2);
            if (p.act == 1) t = gelu2(t);
            if (p.gate) t = __fmul2_rn(t, gate2);
            stg[(2 * i) * STG_PITCH + lane] = t.x;       // token 2i, feature lane
            stg[(2 * i + 1) * STG_PITCH + lane] = t.y;
        }
        __syncwarp();
        const int token = m0 + c * 32 + lane;  // this thread now owns one token row
        // (no early exit here: the next chunk's tcgen05.ld is warp-collective)
        if (token < p.M && nvalid > 0) {
        const float4 *row = reinterpret_cast<const float4 *>(stg + lane * STG_PITCH);
        const int64_t yoff = ((int64_t)p.y_row + token) * p.N + fw;
        if (p.out_f32) {
            float *dst = reinterpret_cast<float *>(p.y) + yoff;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (4 * j >= nvalid) break;
                const float4 v = row[j];
                if (!p.reduce) {
                    *reinterpret_cast<float4 *>(dst + 4 * j) = v;
                } else {
                    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst + 4 * j), "f"(v.x),
                                 "f"(v.y), "f"(v.z), "f"(v.w)
                                 : "memory");
                }
            }
        } else {
            __nv_bfloat16 *dst = reinterpret_cast<__nv_bfloat16 *>(p.y) + yoff;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (8 * j >= nvalid) break;
                const float4 a = row[2 * j], b = row[2 * j + 1];
                const uint4 u = make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(b.x, b.y),
                                           pack_bf16x2(b.z, b.w));
                if (!p.reduce) {
                    *reinterpret_cast<uint4 *>(dst + 8 * j) = u;
                } else {
                    asm volatile("red.global.add.noftz.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(dst + 8 * j),
                                 "r"(u.x), "r"(u.y), "r"(u.z), "r"(u.w)
                                 : "memory");
                }
            }
        }
        }
        __syncwarp();
    }
}

// Flag publication between CTAs of one launch (stream-K partial tiles).
__device__ __forceinline__ void flag_publish(int *flag, int value) {
    asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(flag), "r"(value) : "memory");
}
// Back to 0 once the flag's owner has consumed what it announced; the next
// launch on the stream sees it (kernel boundaries order the store).
__device__ __forceinline__ void flag_clear(int *flag) {
    asm volatile("st.relaxed.gpu.global.b32 [%0], %1;" ::"l"(flag), "r"(0) : "memory");
}
__device__ __forceinline__ int flag_read(const int *flag) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    return v;
}
// Wait until *flag == value, for at most limit_ns; false (and the error word
// set) when the limit expires or another role already failed.
__device__ __forceinline__ bool flag_wait_bounded(const int *flag, int value, int *err, uint64_t limit_ns) {
    if (flag_read(flag) == value) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        __nanosleep(64);
        if (flag_read(flag) == value) return true;
        if (err && *(volatile int *)err != 0) return false;
        if (globaltimer_ns() - t0 > limit_ns) {
            raise_error(err, ERR_WAIT_TIMEOUT);
            return false;
        }
    }
}

}  // namespace lx2v
