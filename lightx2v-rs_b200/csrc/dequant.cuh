// dequant.cuh — device-side decoding of the reference's weight formats.
//
// One "unit" is 16 consecutive values of one weight row, starting at a
// column that is a multiple of 16 and inside one quantization group. A unit
// decodes to 16 f32 products that are bit-identical to the reference's
// dequantize():
//   Q8   q as f32 * s                      crates/lightx2v-core/src/quant.rs:180-186
//   Q4   (c as f32 - z) * s                quant.rs:294-303
//   FP8  e4m3_to_f32(code) * s             quant.rs:409-420, 449-455
// The GEMM rounds these to bf16 (round-to-nearest-even) for the tensor cores;
// the lx2v_weight_dequant_f32 hook writes them out unrounded, so the hook's
// bit-exact test also covers the arithmetic the GEMM uses.
//
// Device layout of a weight (written once at upload, runtime.cu):
//   codes    the reference's own flat code array: Q8 i8 [N*K], FP8 u8 [N*K],
//            Q4 packed nibbles [(N*K+1)/2] (element 2i in the low nibble),
//            native bf16 [N*K];
//   scales   transposed to [G][N] (G = K/group) so that the scales a CTA
//            needs for one k-block are contiguous: f32 for Q8/FP8, and
//            (scale, zero) as a half2 word (low half = scale) for Q4.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace lx2v {

enum : int { FMT_BF16 = 0, FMT_Q8 = 1, FMT_Q4 = 2, FMT_FP8 = 3 };

struct WeightView {
    int fmt;
    int n, k, group;
    const uint8_t *codes;
    const float *scales_t;  // Q8 / FP8: [G][N]
    const uint32_t *sz_t;   // Q4: [G][N], half2 bits (lo = scale, hi = zero)
    int fp8_fast;           // every FP8 scale s satisfies 2^-100 <= s < 2^7
};

// e4m3_to_f32 as the reference defines it (quant.rs:409-420): exponent-field-0
// codes are m/8 * 2^-9 (not the OCP m/8 * 2^-6), 0x7F / 0xFF are NaN.
__device__ __forceinline__ float e4m3_ref(uint32_t code) {
    const float sign = (code & 0x80u) ? -1.0f : 1.0f;
    const uint32_t e = (code >> 3) & 0xFu, m = code & 7u;
    if (e == 0) return sign * ((float)m / 8.0f) * 0x1p-9f;
    if (e == 0xF && m == 7) return __int_as_float(0x7FC00000);
    return sign * (1.0f + (float)m / 8.0f) * __int_as_float((int)((e + 120u) << 23));
}

// Nonzero when some byte of w is zero.
__device__ __forceinline__ uint32_t has_zero_byte(uint32_t w) {
    return (w - 0x01010101u) & ~w & 0x80808080u;
}

// ---- Q8 -----------------------------------------------------------------
// 16 int8 codes (one uint4) times scale s. The code is turned into an exact
// f32 with the 2^23 magic number: bits 0x4B0000xx = 2^23 + xx, xx = q + 128.
__device__ __forceinline__ void dq_q8_unit(const uint4 raw, float s, float (&out)[16]) {
    const uint32_t w[4] = {raw.x ^ 0x80808080u, raw.y ^ 0x80808080u, raw.z ^ 0x80808080u,
                           raw.w ^ 0x80808080u};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float q = __int_as_float((int)__byte_perm(w[j], 0x4B000000u, 0x7440u + i)) -
                            8388736.0f;  // 2^23 + 128
            out[4 * j + i] = q * s;
        }
    }
}

// ---- FP8 (reference e4m3) -----------------------------------------------
// Fast path for a unit without exponent-field-0 or NaN codes and with a
// scale in the fast range: a code's low 7 bits shifted to bit 20 are the
// f32 bit pattern of |value| * 2^-120, so |value| * s = that float *
// (s * 2^120), one correctly rounded multiply of the same real product.
// The sign is then copied in from the code's bit 7.
__device__ __forceinline__ void dq_fp8_unit(const uint4 raw, float s, bool fast_scale,
                                            float (&out)[16]) {
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
    uint32_t special = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        special |= has_zero_byte(w[j] & 0x78787878u);      // exponent field 0
        special |= has_zero_byte(~w[j] & 0x7F7F7F7Fu);     // 0x7F / 0xFF (NaN)
    }
    if (special == 0 && fast_scale) {
        const float s120 = s * 0x1p120f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t c = (w[j] >> (8 * i)) & 0xFFu;
                const float mag = __int_as_float((int)((c & 0x7Fu) << 20)) * s120;
                out[4 * j + i] = __int_as_float(__float_as_int(mag) ^ (int)((c & 0x80u) << 24));
            }
        }
    } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
#pragma unroll
            for (int i = 0; i < 4; ++i) out[4 * j + i] = e4m3_ref((w[j] >> (8 * i)) & 0xFFu) * s;
        }
    }
}

// ---- Q4 -----------------------------------------------------------------
// 16 nibbles (one uint2; element 2i in the low nibble) with f16-exact scale
// s and zero z: (c - z) * s, two roundings as the reference does them.
__device__ __forceinline__ void dq_q4_unit(const uint2 raw, float s, float z, float (&out)[16]) {
    const uint32_t w[2] = {raw.x, raw.y};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t c = (w[j] >> (4 * i)) & 0xFu;
            const float cf = __int_as_float((int)(0x4B000000u | c)) - 8388608.0f;
            out[8 * j + i] = (cf - z) * s;
        }
    }
}

__device__ __forceinline__ void q4_scale_zero(uint32_t sz, float &s, float &z) {
    const __half2 h = *reinterpret_cast<const __half2 *>(&sz);
    s = __low2float(h);
    z = __high2float(h);
}

// ---- generic element access (any shape) ---------------------------------
// Flat element i = n*K + k of the reference's code array; group index is
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
        default:
            return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(w.codes)[i]);
    }
}

// Whether the 16-value unit path applies: rows start 16-byte aligned, units
// never straddle a group.
__host__ __device__ inline bool unit_path_ok(int fmt, int k, int group) {
    if (group % 16 != 0) return false;
    switch (fmt) {
        case FMT_Q8:
        case FMT_FP8: return k % 16 == 0;
        case FMT_Q4: return k % 32 == 0;
        default: return k % 8 == 0;
    }
}

// Decode the unit of row n starting at column k0 (k0 % 16 == 0, k0 < K).
__device__ __forceinline__ void dq_unit(const WeightView &w, int n, int k0, float (&out)[16]) {
    const int64_t base = (int64_t)n * w.k + k0;
    const int64_t g = k0 / w.group;
    switch (w.fmt) {
        case FMT_Q8: {
            const uint4 raw = *reinterpret_cast<const uint4 *>(w.codes + base);
            dq_q8_unit(raw, w.scales_t[g * w.n + n], out);
            break;
        }
        case FMT_FP8: {
            const uint4 raw = *reinterpret_cast<const uint4 *>(w.codes + base);
            dq_fp8_unit(raw, w.scales_t[g * w.n + n], w.fp8_fast != 0, out);
            break;
        }
        case FMT_Q4: {
            const uint2 raw = *reinterpret_cast<const uint2 *>(w.codes + base / 2);
            float s, z;
            q4_scale_zero(w.sz_t[g * w.n + n], s, z);
            dq_q4_unit(raw, s, z, out);
            break;
        }
        default: {
            const __nv_bfloat16 *p = reinterpret_cast<const __nv_bfloat16 *>(w.codes) + base;
#pragma unroll
            for (int i = 0; i < 16; ++i) out[i] = __bfloat162float(p[i]);
        }
    }
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&v);
}

}  // namespace lx2v
