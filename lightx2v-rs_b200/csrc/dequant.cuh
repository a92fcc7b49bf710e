// dequant.cuh — device-side decoding of the reference's weight formats.
//
// One "unit" is 16 consecutive values of one weight row, starting at a
// column that is a multiple of 16 and inside one quantization group. A unit
// decodes to 16 f32 products that are bit-identical to the reference's
// dequantize():
//   Q8   q as f32 * s                      crates/lightx2v-core/src/quant.rs:180-186
//   Q4   (c as f32 - z) * s                quant.rs:294-303
//   FP8  e4m3_to_f32(code) * s             quant.rs:409-420, 449-455
// The GEMM rounds each product to bf16 (round-to-nearest-even) for the tensor
// cores; the lx2v_weight_dequant_f32 hook runs the same decode functions and
// writes the products unrounded, so its bit-exact test covers the GEMM's
// arithmetic too.
//
// Products are formed two at a time with the sm_100 packed f32 multiply
// (__fmul2_rn: two independent IEEE round-to-nearest multiplies).
//
// Device layout of a weight (written once at upload, runtime.cu):
//   codes    the reference's own flat code array: Q8 i8 [N*K], FP8 u8 [N*K],
//            Q4 packed nibbles [(N*K+1)/2] (element 2i in the low nibble),
//            native bf16 [N*K];
//   scales   transposed to [G][N] (G = K/group) so that the scales of one
//            k-block are contiguous across rows: f32 for Q8/FP8, and
//            (scale, zero) as a half2 word (low half = scale) for Q4;
//   flags    FP8 only, one byte per (32-column block, row), stored [K/32][N]
//            so one k-block's flags are contiguous across rows: 0 = fast decode;
//            1 = the block holds a code the fast decode does not cover (an
//            exponent-field-0 code, a NaN code 0x7F/0xFF) and takes the fast
//            decode plus an exact fix-up; 2 = a scale outside [2^-100, 2^7),
//            the block takes the reference formula.
#pragma once
#include <cstdint>
#include <cstring>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace lx2v {

enum : int { FMT_BF16 = 0, FMT_Q8 = 1, FMT_Q4 = 2, FMT_FP8 = 3, FMT_NVFP4 = 4 };

struct WeightView {
    int fmt;
    int n, k, group;
    const uint8_t *codes;
    const float *scales_t;  // Q8 / FP8: [G][N]; NVFP4: [K/16][N] effective scales (block e4m3 x global)
    const uint32_t *sz_t;   // Q4: [G][N], half2 bits (lo = scale, hi = zero)
    const uint8_t *flags;   // FP8: [ceil(K/32)][N]
};

__host__ __device__ inline int fp8_flag_cols(int k) { return (k + 31) / 32; }

// e4m3_to_f32 as the reference defines it (quant.rs:409-420): exponent-field-0
// codes are m/8 * 2^-9 (not the OCP m/8 * 2^-6), 0x7F / 0xFF are NaN.
__host__ __device__ inline float e4m3_ref(uint32_t code) {
    const float sign = (code & 0x80u) ? -1.0f : 1.0f;
    const uint32_t e = (code >> 3) & 0xFu, m = code & 7u;
    if (e == 0) return sign * ((float)m / 8.0f) * 0x1p-9f;
    if (e == 0xF && m == 7) {
        const uint32_t nan_bits = 0x7FC00000u;
        float f;
        memcpy(&f, &nan_bits, 4);
        return f;
    }
    uint32_t bits = (e + 120u) << 23;
    float p2;
    memcpy(&p2, &bits, 4);
    return sign * (1.0f + (float)m / 8.0f) * p2;
}

// Whether a code needs the reference formula (exponent field 0 or NaN).
__host__ __device__ inline bool fp8_code_special(uint32_t c) {
    return ((c & 0x78u) == 0) || ((c & 0x7Fu) == 0x7Fu);
}
__host__ __device__ inline bool fp8_scale_fast(float s) { return s >= 0x1p-100f && s < 0x1p7f; }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&v);
}
__device__ __forceinline__ uint32_t pack_bf16x2(float2 v) { return pack_bf16x2(v.x, v.y); }

// ---- Q8 -----------------------------------------------------------------
// 16 int8 codes (one uint4) times scale s: p[i] = (q_{2i} * s, q_{2i+1} * s).
// A code becomes an exact f32 with the 2^23 magic number: the bit pattern
// 0x4B0000xx is 2^23 + xx, and xx = q + 128.
__device__ __forceinline__ void q8_products(const uint4 raw, float s, float2 (&p)[8]) {
    const uint32_t w[4] = {raw.x ^ 0x80808080u, raw.y ^ 0x80808080u, raw.z ^ 0x80808080u,
                           raw.w ^ 0x80808080u};
    const float2 off = make_float2(-8388736.0f, -8388736.0f);  // -(2^23 + 128)
    const float2 s2 = make_float2(s, s);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float2 q;
            q.x = __int_as_float((int)__byte_perm(w[j], 0x4B000000u, 0x7440u + 2 * h));
            q.y = __int_as_float((int)__byte_perm(w[j], 0x4B000000u, 0x7441u + 2 * h));
            p[2 * j + h] = __fmul2_rn(__fadd2_rn(q, off), s2);
        }
    }
}

// ---- FP8 (reference e4m3) -----------------------------------------------
// Fast path, for a unit without special codes and with a fast-range scale: a
// code's low 7 bits shifted to bit 20 are the f32 bit pattern of
// |value| * 2^-120, so |value| * s = that float * (s * 2^120), one correctly
// rounded multiply of the same real product. Returns the magnitudes; the
// signs (code bit 7) are applied after rounding, which commutes with it.
__device__ __forceinline__ void fp8_magnitudes(const uint4 raw, float s, float2 (&p)[8]) {
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
    const float s120 = s * 0x1p120f;
    const float2 s2 = make_float2(s120, s120);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float2 a, b;
        a.x = __uint_as_float((w[j] << 20) & 0x07F00000u);
        a.y = __uint_as_float((w[j] << 12) & 0x07F00000u);
        b.x = __uint_as_float((w[j] << 4) & 0x07F00000u);
        b.y = __uint_as_float((w[j] >> 4) & 0x07F00000u);
        p[2 * j] = __fmul2_rn(a, s2);
        p[2 * j + 1] = __fmul2_rn(b, s2);
    }
}
// Sign bits of codes 2i, 2i+1 placed at bits 15 and 31 (a bf16x2 sign mask).
__device__ __forceinline__ uint32_t fp8_sign_pair_bf16(const uint4 raw, int i) {
    const uint32_t w = (i < 2) ? raw.x : (i < 4) ? raw.y : (i < 6) ? raw.z : raw.w;
    return __byte_perm(w, 0u, (i & 1) ? 0x3424u : 0x1404u) & 0x80008000u;
}
// Fix-up of fast-path products (fp8_magnitudes or fp8_products_hw) for a
// block that holds special codes (its scale is in the fast range): an
// exponent-field-0 code m decodes to m/8 * 2^-9 (quant.rs:413-414) but both
// fast decoders give m * 2^-9, so the product is scaled by 2^-3 (exact: the
// fast product is at least 2^-109 in magnitude or zero); the NaN codes
// 0x7F / 0xFF become NaN.
__device__ __forceinline__ void fp8_fixup(const uint4 raw, float2 (&p)[8]) {
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
    const float qnan = __uint_as_float(0x7FC00000u);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const uint32_t c = (w[i >> 2] >> (8 * (i & 3))) & 0xFFu;
        float v = (i & 1) ? p[i >> 1].y : p[i >> 1].x;
        v = ((c & 0x78u) == 0) ? v * 0.125f : v;
        v = ((c & 0x7Fu) == 0x7Fu) ? qnan : v;
        if (i & 1) p[i >> 1].y = v; else p[i >> 1].x = v;
    }
}

// Signed products with the hardware e4m3 converter: cvt.rn.f16x2.e4m3x2
// gives the exact IEEE-style e4m3 value as f16 (f16 holds every e4m3 value,
// subnormals included), the f16 -> f32 widening is exact, and one f32
// multiply rounds decode(c) * s exactly as the reference does
// (quant.rs:400-420). IEEE-style decoding differs from the reference only on
// exponent-field-0 codes (2^3 larger) and on 0x7F / 0xFF, which fp8_fixup
// corrects in blocks the upload flagged; it needs no restriction on s.
__device__ __forceinline__ void fp8_products_hw(const uint4 raw, float s, float2 (&p)[8]) {
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
    const float2 s2 = make_float2(s, s);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t h0, h1;
        asm("{\n\t.reg .b16 lo, hi;\n\t"
            "mov.b32 {lo, hi}, %2;\n\t"
            "cvt.rn.f16x2.e4m3x2 %0, lo;\n\t"
            "cvt.rn.f16x2.e4m3x2 %1, hi;\n\t}"
            : "=r"(h0), "=r"(h1)
            : "r"(w[j]));
        const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&h0));
        const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&h1));
        p[2 * j] = __fmul2_rn(f0, s2);
        p[2 * j + 1] = __fmul2_rn(f1, s2);
    }
}

// Reference-formula path: signed products.
__device__ __forceinline__ void fp8_products_slow(const uint4 raw, float s, float2 (&p)[8]) {
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        p[2 * j] = make_float2(e4m3_ref(w[j] & 0xFFu) * s, e4m3_ref((w[j] >> 8) & 0xFFu) * s);
        p[2 * j + 1] = make_float2(e4m3_ref((w[j] >> 16) & 0xFFu) * s, e4m3_ref(w[j] >> 24) * s);
    }
}

// ---- Q4 -----------------------------------------------------------------
// 16 nibbles (one uint2; element 2i in the low nibble) with f16-exact scale
// s and zero z: (c - z) * s with the reference's two roundings.
__device__ __forceinline__ void q4_products(const uint2 raw, float s, float z, float2 (&p)[8]) {
    const uint32_t w[2] = {raw.x, raw.y};
    const float2 m23 = make_float2(-8388608.0f, -8388608.0f);
    const float2 nz = make_float2(-z, -z), s2 = make_float2(s, s);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        // low and high nibbles of the four bytes, then one byte permute per
        // value builds the float 2^23 + c (byte 3 = 0x4B, byte 0 = c)
        const uint32_t lo = w[j] & 0x0F0F0F0Fu, hi = (w[j] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float2 c;
            c.x = __uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7650u | (uint32_t)i));
            c.y = __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7650u | (uint32_t)i));
            p[4 * j + i] = __fmul2_rn(__fadd2_rn(__fadd2_rn(c, m23), nz), s2);
        }
    }
}

// NVFP4 (fp4 e2m1 codes, one e4m3 scale per 16 values, one f32 global scale;
// no counterpart in the reference, which names it as its next quantisation):
// a code's value {0, 0.5, 1, 1.5, 2, 3, 4, 6} (bit 3 the sign), built as an
// f32 bit pattern; the weight is value x (block scale x global scale), the
// bracket formed in f32 once per block at upload.
__host__ __device__ __forceinline__ float e2m1_value(uint32_t c) {
    const uint32_t m = c & 7u;
    const uint32_t bits = m < 2u ? (m ? 0x3F000000u : 0u) : ((((m >> 1) + 126u) << 23) | ((m & 1u) << 22));
    const uint32_t v = bits | ((c & 8u) << 28);
    float f;
    memcpy(&f, &v, 4);
    return f;
}
// 16 packed codes (element 2i in the low nibble, as Q4 packs them) -> value x s.
__device__ __forceinline__ void nvfp4_products(const uint2 raw, float s, float2 (&p)[8]) {
    const uint32_t w[2] = {raw.x, raw.y};
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t b = (w[j] >> (8 * i)) & 0xFFu;
            p[4 * j + i] = make_float2(e2m1_value(b & 0xFu) * s, e2m1_value(b >> 4) * s);
        }
}

__device__ __forceinline__ void q4_scale_zero(uint32_t sz, float &s, float &z) {
    const __half2 h = *reinterpret_cast<const __half2 *>(&sz);
    s = __low2float(h);
    z = __high2float(h);
}

// ---- one unit, f32 out (hook) or bf16x2 out (GEMM) ---------------------------
// `raw` holds the unit's codes: 16 bytes (Q8/FP8), 8 bytes in .x/.y (Q4),
// or 32 bytes of bf16 split over raw/raw2 (native).
// fp8_mode: 0 fast, 1 fast + special-code fix-up, 2 reference formula.
// The FP8 units of blocks that hold special codes or extreme scales (modes 1
// and 2), out of line: they are rare, and keeping their code out of the
// decode loop keeps that loop small for the instruction cache that the
// kernel's other warps share.
struct PackedUnit {
    uint32_t w[8];
};
static __device__ __noinline__ PackedUnit fp8_unit_special(const uint4 raw, float s, int fp8_mode) {
    float2 p[8];
    if (fp8_mode == 1) {
        fp8_products_hw(raw, s, p);
        fp8_fixup(raw, p);
    } else {
        fp8_products_slow(raw, s, p);
    }
    PackedUnit u;
#pragma unroll
    for (int i = 0; i < 8; ++i) u.w[i] = pack_bf16x2(p[i]);
    return u;
}

template <int FMT>
__device__ __forceinline__ void unit_to_bf16(const uint4 raw, const uint4 raw2, float s, float z,
                                             int fp8_mode, uint32_t (&out)[8]) {
    if (FMT == FMT_BF16) {
        out[0] = raw.x; out[1] = raw.y; out[2] = raw.z; out[3] = raw.w;
        out[4] = raw2.x; out[5] = raw2.y; out[6] = raw2.z; out[7] = raw2.w;
        return;
    }
    float2 p[8];
    if (FMT == FMT_Q8) {
        q8_products(raw, s, p);
    } else if (FMT == FMT_Q4) {
        q4_products(make_uint2(raw.x, raw.y), s, z, p);
    } else if (FMT == FMT_NVFP4) {
        nvfp4_products(make_uint2(raw.x, raw.y), s, p);
    } else {
        if (fp8_mode != 0) {
            const PackedUnit u = fp8_unit_special(raw, s, fp8_mode);
#pragma unroll
            for (int i = 0; i < 8; ++i) out[i] = u.w[i];
            return;
        }
        fp8_products_hw(raw, s, p);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = pack_bf16x2(p[i]);
}

template <int FMT>
__device__ __forceinline__ void unit_to_f32(const uint4 raw, float s, float z, int fp8_mode,
                                            float (&out)[16]) {
    float2 p[8];
    if (FMT == FMT_Q8) {
        q8_products(raw, s, p);
    } else if (FMT == FMT_Q4) {
        q4_products(make_uint2(raw.x, raw.y), s, z, p);
    } else if (FMT == FMT_NVFP4) {
        nvfp4_products(make_uint2(raw.x, raw.y), s, p);
    } else {
        if (fp8_mode != 2) {
            fp8_magnitudes(raw, s, p);
            if (fp8_mode == 1) fp8_fixup(raw, p);
            const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const uint32_t sign = ((w[i >> 2] >> (8 * (i & 3))) & 0x80u) << 24;
                const float mag = (i & 1) ? p[i >> 1].y : p[i >> 1].x;
                out[i] = __uint_as_float(__float_as_uint(mag) ^ sign);
            }
            return;
        }
        fp8_products_slow(raw, s, p);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) { out[2 * i] = p[i].x; out[2 * i + 1] = p[i].y; }
}

// ---- generic element access (any shape) ---------------------------------
// Flat element i = n*K + k of the reference's code array; the group index is
// i / group over the flat array, which equals n * (K/group) + k/group.
__device__ __forceinline__ float dq_elem(const WeightView &w, int64_t n, int64_t k) {
    const int64_t i = n * (int64_t)w.k + k;
    const int64_t g = k / w.group;
    switch (w.fmt) {
        case FMT_Q8:
            return (float)(int8_t)w.codes[i] * w.scales_t[g * w.n + n];
        case FMT_FP8:
            return e4m3_ref(w.codes[i]) * w.scales_t[g * w.n + n];
        case FMT_Q4: {
            float s, z;
            q4_scale_zero(w.sz_t[g * w.n + n], s, z);
            const uint32_t c = (w.codes[i >> 1] >> (4 * (i & 1))) & 0xFu;
            return ((float)c - z) * s;
        }
        case FMT_NVFP4:
            return e2m1_value((w.codes[i >> 1] >> (4 * (i & 1))) & 0xFu) * w.scales_t[g * w.n + n];
        default:
            return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(w.codes)[i]);
    }
}

// Whether the 16-value unit path applies: rows start 16-byte aligned and a
// unit never straddles a group.
__host__ __device__ inline bool unit_path_ok(int fmt, int k, int group) {
    if (group % 16 != 0) return false;
    switch (fmt) {
        case FMT_Q8:
        case FMT_FP8: return k % 16 == 0;
        case FMT_Q4:
        case FMT_NVFP4: return k % 32 == 0;
        default: return k % 8 == 0;
    }
}

}  // namespace lx2v
