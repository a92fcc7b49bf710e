/*
 * lx2v_oracle.c — CPU restatement of lightx2v-rs's quantized-linear path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the parity checker for the CUDA
 * library in lightx2v-rs_b200/. Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py load it. The product path never
 * links or calls it.
 *
 * Every function restates one function of the Rust reference. The citation
 * is given as crates/<crate>/src/<file>.rs:<line>. The arithmetic is kept
 * operation-for-operation:
 *   - all float math is f32, evaluated left to right as the Rust source
 *     writes it. The build uses -ffp-contract=off, because rustc never fuses
 *     a*b+c into an FMA;
 *   - the transcendental calls (logf, log2f, sqrtf, cosf, sinf, powf, tanhf)
 *     go to the same glibc libm that Rust's std calls on Linux;
 *   - f32 -> f16 rounding (the `half` 2.7.1 crate, pinned in Cargo.lock) is
 *     IEEE round-to-nearest-even, done here with GCC's _Float16.
 * Parity of libm and `half` is not pinned by any reference test. The
 * reference's own known-answer tests (e4m3 spot values, the check_linear
 * hand case, the quantizer error bounds, check_quant) are run against this
 * file in tests/test_oracle.py.
 */
#include <math.h>
#include <stdint.h>
#include <stddef.h>
#include <string.h>
#include <stdlib.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define Q8_GROUP 128      /* quant.rs:19 */
#define FP8_GROUP 128     /* quant.rs:21 */
#define FP8_E4M3_MAX 448.0f /* quant.rs:23 */
#define PI_F32 3.14159265358979323846f

/* ---------------------------------------------------------------- rng ---- */
/* Rng, crates/lightx2v-core/src/rng.rs:8-53 (SplitMix64 + Box-Muller). */
typedef struct { uint64_t state; } orc_rng;

void orc_rng_init(orc_rng *r, uint64_t seed) {
    r->state = seed + 0x9E3779B97F4A7C15ULL; /* rng.rs:13-18 */
}

static uint64_t rng_next_u64(orc_rng *r) { /* rng.rs:20-26 */
    r->state += 0x9E3779B97F4A7C15ULL;
    uint64_t z = r->state;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

static float rng_next_f32(orc_rng *r) { /* rng.rs:29-31 */
    return (float)(rng_next_u64(r) >> 40) / (float)(1ULL << 24);
}

void orc_rng_uniform(orc_rng *r, size_t n, float a, float *out) { /* rng.rs:34-36 */
    for (size_t i = 0; i < n; i++) out[i] = (rng_next_f32(r) * 2.0f - 1.0f) * a;
}

void orc_rng_normal(orc_rng *r, size_t n, float *out) { /* rng.rs:39-52 */
    size_t len = 0;
    while (len < n) {
        float u1 = rng_next_f32(r);
        u1 = fmaxf(u1, 1e-7f);
        float u2 = rng_next_f32(r);
        float rr = sqrtf(-2.0f * logf(u1));
        float t = 2.0f * PI_F32 * u2;
        out[len++] = rr * cosf(t);
        if (len < n) out[len++] = rr * sinf(t);
    }
}

/* Convenience used by the tests and the bench: a fresh Rng(seed).normal(n)
 * scaled by `std` (the BASELINE inputs are `std * normal`). */
void orc_normal(uint64_t seed, size_t n, float std_, float *out) {
    orc_rng r;
    orc_rng_init(&r, seed);
    orc_rng_normal(&r, n, out);
    if (std_ != 1.0f)
        for (size_t i = 0; i < n; i++) out[i] = out[i] * std_;
}

void orc_uniform(uint64_t seed, size_t n, float a, float *out) {
    orc_rng r;
    orc_rng_init(&r, seed);
    orc_rng_uniform(&r, n, a, out);
}

/* -------------------------------------------------------------- quant ---- */
/* Rust f32::max / f32::min ignore a NaN operand, like fmaxf / fminf. */
static float rust_round(float v) { return roundf(v); } /* half away from 0 */

/* Rust `f as i8` / `f as u8`: saturating, NaN -> 0. */
static int8_t sat_i8(float v) {
    if (v != v) return 0;
    if (v >= 127.0f) return 127;
    if (v <= -128.0f) return -128;
    return (int8_t)v;
}
static uint8_t sat_u8(float v) {
    if (v != v) return 0;
    if (v >= 255.0f) return 255;
    if (v <= 0.0f) return 0;
    return (uint8_t)v;
}
static float rust_clamp(float v, float lo, float hi) { /* f32::clamp keeps NaN */
    if (v < lo) v = lo;
    if (v > hi) v = hi;
    return v;
}

/* Q8::quantize, quant.rs:154-178. Returns the group used. */
size_t orc_q8_quantize(const float *data, size_t rows, size_t cols,
                       int8_t *q, float *scales) {
    size_t group = (cols % Q8_GROUP == 0) ? Q8_GROUP : cols;
    size_t n = rows * cols;
    for (size_t g0 = 0, gi = 0; g0 < n; g0 += group, gi++) {
        float amax = 0.0f;
        for (size_t i = 0; i < group; i++) amax = fmaxf(amax, fabsf(data[g0 + i]));
        float s = amax > 0.0f ? amax / 127.0f : 1.0f;
        for (size_t i = 0; i < group; i++)
            q[g0 + i] = sat_i8(rust_clamp(rust_round(data[g0 + i] / s), -127.0f, 127.0f));
        scales[gi] = s;
    }
    return group;
}

/* Q8::dequantize, quant.rs:180-186. */
void orc_q8_dequantize(const int8_t *q, const float *scales, size_t n,
                       size_t group, float *out) {
    for (size_t i = 0; i < n; i++) out[i] = (float)q[i] * scales[i / group];
}

static float f16_round(float v) { return (float)(_Float16)v; } /* half::f16::from_f32 */

/* Q4::quantize, quant.rs:226-292 (RTN, optional HQQ zero refinement).
 * Returns the group used. `q` gets one code per byte. */
size_t orc_q4_quantize(const float *data, size_t rows, size_t cols, size_t group,
                       int hqq, uint8_t *q, float *scales, float *zeros) {
    if (cols % group != 0) group = cols; /* quant.rs:228-232 */
    size_t n = rows * cols;
    for (size_t g0 = 0, gi = 0; g0 < n; g0 += group, gi++) {
        const float *w = data + g0;
        float lo = 3.40282347e+38f, hi = -3.40282347e+38f;
        for (size_t i = 0; i < group; i++) { lo = fminf(lo, w[i]); hi = fmaxf(hi, w[i]); }
        float is = hi > lo ? 15.0f / (hi - lo) : 1.0f;
        float z = -lo * is;
#define Q4_CODE(v, zz) rust_clamp(rust_round((v) * is + (zz)), 0.0f, 15.0f)
        if (hqq) { /* quant.rs:248-276 */
            float p = 0.7f, beta = 10.0f, kappa = 1.01f;
            float best = 3.40282347e+38f, best_z = z;
            for (int it = 0; it < 20; it++) {
                float err = 0.0f, zsum = 0.0f;
                for (size_t i = 0; i < group; i++) {
                    float v = w[i];
                    float c = Q4_CODE(v, z);
                    float r = (c - z) / is;
                    float e = v - r;
                    err += fabsf(e);
                    float a = fabsf(e);
                    float sh;
                    if (a > 0.0f) {
                        float t = a - powf(a, p - 1.0f) / beta;
                        t = fmaxf(t, 0.0f);
                        float sg = (e > 0.0f) ? 1.0f : -1.0f; /* e.signum(), e != 0 here */
                        sh = sg * t;
                    } else {
                        sh = 0.0f;
                    }
                    zsum += c - (v - sh) * is;
                }
                err = err / (float)group;
                if (err >= best) break;
                best = err;
                best_z = z;
                z = zsum / (float)group;
                beta *= kappa;
            }
            z = best_z;
        }
        for (size_t i = 0; i < group; i++) q[g0 + i] = sat_u8(Q4_CODE(w[i], z));
#undef Q4_CODE
        scales[gi] = f16_round(1.0f / is);
        zeros[gi] = f16_round(z);
    }
    return group;
}

/* Q4::dequantize, quant.rs:294-303 (one code per byte). */
void orc_q4_dequantize(const uint8_t *q, const float *scales, const float *zeros,
                       size_t n, size_t group, float *out) {
    for (size_t i = 0; i < n; i++) {
        size_t g = i / group;
        out[i] = ((float)q[i] - zeros[g]) * scales[g];
    }
}

/* Q4::packed, quant.rs:306-311: element 2i in the low nibble. */
void orc_q4_pack(const uint8_t *q, size_t n, uint8_t *packed) {
    for (size_t i = 0; i < n; i += 2) {
        uint8_t lo = q[i], hi = (i + 1 < n) ? q[i + 1] : 0;
        packed[i / 2] = (uint8_t)(lo | (uint8_t)(hi << 4));
    }
}

/* Q4::from_packed, quant.rs:313-336 (codes only). */
void orc_q4_unpack(const uint8_t *packed, size_t n, uint8_t *q) {
    for (size_t i = 0; i < n; i++) q[i] = (packed[i / 2] >> (4 * (i % 2))) & 15;
}

/* f32_to_e4m3, quant.rs:376-406, restated with its small-magnitude defect:
 * for e in {-8, -7... } the `(e + 7) as u8` cast wraps for e < -7, and the
 * u8 shift `exp << 3` drops the high bits, exactly as Rust does. */
uint8_t orc_f32_to_e4m3(float v) {
    if (v == 0.0f) return signbit(v) ? 0x80 : 0x00;
    uint8_t sign = signbit(v) ? 0x80 : 0x00;
    float a = fabsf(v);
    if (!isfinite(a) || a >= 464.0f) return sign | 0x7E;
    float lf = floorf(log2f(a));
    int e;
    if (lf != lf) e = 0; /* unreachable for finite a > 0 */
    else if (lf <= -2147483648.0f) e = INT32_MIN;
    else if (lf >= 2147483647.0f) e = INT32_MAX;
    else e = (int)lf;
    if (e < -9) {
        float m = rust_round(a / (ldexpf(1.0f, -9) / 8.0f));
        uint8_t mm = sat_u8(m);
        return sign | (mm < 7 ? mm : 7);
    }
    if (e > 8) return sign | 0x7E;
    uint8_t exp = (uint8_t)(e + 7);           /* wraps like `as u8` */
    uint8_t mant = sat_u8(rust_round((a / ldexpf(1.0f, e) - 1.0f) * 8.0f));
    if (mant >= 8) {
        if (exp >= 15) return sign | 0x7E;
        return sign | (uint8_t)((uint8_t)(exp + 1) << 3);
    }
    return sign | (uint8_t)(exp << 3) | mant;
}

/* e4m3_to_f32, quant.rs:409-420: exponent-field-0 codes decode as m/8*2^-9. */
float orc_e4m3_to_f32(uint8_t code) {
    float sign = (code & 0x80) ? -1.0f : 1.0f;
    unsigned exp = (code >> 3) & 0xF, mant = code & 0x7;
    if (exp == 0) return sign * ((float)mant / 8.0f) * ldexpf(1.0f, -9);
    if (exp == 0xF && mant == 0x7) return NAN;
    return sign * (1.0f + (float)mant / 8.0f) * ldexpf(1.0f, (int)exp - 7);
}

/* Fp8E4M3::quantize, quant.rs:423-447. Returns the group used. */
size_t orc_fp8_quantize(const float *data, size_t rows, size_t cols,
                        uint8_t *q, float *scales) {
    size_t group = (cols % FP8_GROUP == 0) ? FP8_GROUP : cols;
    size_t n = rows * cols;
    for (size_t g0 = 0, gi = 0; g0 < n; g0 += group, gi++) {
        float amax = 0.0f;
        for (size_t i = 0; i < group; i++) amax = fmaxf(amax, fabsf(data[g0 + i]));
        float s = amax > 0.0f ? amax / FP8_E4M3_MAX : 1.0f;
        for (size_t i = 0; i < group; i++) q[g0 + i] = orc_f32_to_e4m3(data[g0 + i] / s);
        scales[gi] = s;
    }
    return group;
}

/* Fp8E4M3::dequantize, quant.rs:449-455. */
void orc_fp8_dequantize(const uint8_t *q, const float *scales, size_t n,
                        size_t group, float *out) {
    for (size_t i = 0; i < n; i++) out[i] = orc_e4m3_to_f32(q[i]) * scales[i / group];
}

/* ------------------------------------------------------------- linear ---- */
/* gelu_tanh, crates/lightx2v-cpu/src/lib.rs:151-153. */
float orc_gelu_tanh(float x) {
    float c = sqrtf(2.0f / PI_F32);
    return 0.5f * x * (1.0f + tanhf(c * (x + 0.044715f * x * x * x)));
}

/* CpuBackend::linear, crates/lightx2v-cpu/src/lib.rs:296-326:
 *   y[(y_row + r) * N + o] = act(sum_i x[(x_row + r) * K + i] * w[o * K + i] + b[o])
 * with a sequential f32 accumulation over i. `w` is the dequantized f32
 * matrix [N, K] (weight_q8/q4/fp8 dequantize first, lib.rs:259-284).
 * `threads` > 1 splits the rows over OpenMP threads; each output element is
 * still the same sequential loop, so the result does not depend on it. */
void orc_linear(const float *x, size_t x_row, size_t rows, const float *w,
                size_t n_out, size_t k, const float *bias, int act, float *y,
                size_t y_row, int threads) {
#ifdef _OPENMP
    int nt = threads > 0 ? threads : 1;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nt)
#endif
    for (long long r = 0; r < (long long)rows; r++) {
        const float *xr = x + (x_row + (size_t)r) * k;
        float *yr = y + (y_row + (size_t)r) * n_out;
        for (size_t o = 0; o < n_out; o++) {
            const float *wo = w + o * k;
            float acc = 0.0f;
            for (size_t i = 0; i < k; i++) acc += xr[i] * wo[i];
            if (bias) acc += bias[o];
            yr[o] = act == 1 ? orc_gelu_tanh(acc) : acc;
        }
    }
}

/* CpuBackend::gate_residual, crates/lightx2v-cpu/src/lib.rs:394-404:
 *   h[r * dim + j] += a[r * dim + j] * mods[gate * dim + j] */
void orc_gate_residual(float *h, const float *a, size_t rows, size_t dim,
                       const float *mods, size_t gate) {
    for (size_t r = 0; r < rows; r++)
        for (size_t j = 0; j < dim; j++)
            h[r * dim + j] += a[r * dim + j] * mods[gate * dim + j];
}

/* ---------------------------------------------------------- attention ---- */
/* softmax_row, crates/lightx2v-cpu/src/lib.rs:155-166: max by f32::max
 * (NaN-ignoring, fmaxf), exp of the shifted scores, sequential sum, then a
 * multiply by the reciprocal. */
static void orc_softmax_row(float *s, size_t n) {
    float m = -INFINITY;
    for (size_t i = 0; i < n; i++) m = fmaxf(m, s[i]);
    float sum = 0.0f;
    for (size_t i = 0; i < n; i++) {
        s[i] = expf(s[i] - m);
        sum += s[i];
    }
    float inv = 1.0f / sum;
    for (size_t i = 0; i < n; i++) s[i] *= inv;
}

/* attention_impl, crates/lightx2v-cpu/src/lib.rs:170-208 (both
 * CpuBackend::attention and causal_attention, lib.rs:462-494): q is
 * [heads, sq, d], k / v [heads, sk, d], mask [sq, sk] (nonzero = allowed) or
 * NULL, out [sq, heads * d]. Scores are sequential-d dot products times
 * 1/sqrt(d); a forbidden pair scores -inf. `threads` > 1 spreads the
 * (head, query) rows over OpenMP threads; each row is computed exactly as
 * the reference computes it. */
void orc_attention(const float *q, const float *k, const float *v, size_t heads, size_t sq, size_t sk,
                   size_t d, const uint8_t *mask, float *out, int threads) {
    const float scale = 1.0f / sqrtf((float)d);
#ifdef _OPENMP
    int nt = threads > 0 ? threads : 1;
#pragma omp parallel num_threads(nt)
#endif
    {
        float *scores = (float *)malloc(sk * sizeof(float));
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (long long row = 0; row < (long long)(heads * sq); row++) {
            const size_t h = (size_t)row / sq, qi = (size_t)row % sq;
            for (size_t ki = 0; ki < sk; ki++) {
                if (mask && !mask[qi * sk + ki]) {
                    scores[ki] = -INFINITY;
                    continue;
                }
                float acc = 0.0f;
                for (size_t j = 0; j < d; j++) acc += q[(h * sq + qi) * d + j] * k[(h * sk + ki) * d + j];
                scores[ki] = acc * scale;
            }
            orc_softmax_row(scores, sk);
            for (size_t j = 0; j < d; j++) {
                float acc = 0.0f;
                for (size_t ki = 0; ki < sk; ki++) acc += scores[ki] * v[(h * sk + ki) * d + j];
                out[(qi * heads + h) * d + j] = acc;
            }
        }
        free(scores);
    }
}

/* ------------------------------------------------------------- norms ---- */
/* CpuBackend::layer_norm, crates/lightx2v-cpu/src/lib.rs:328-362. kind 0 =
 * NormKind::Affine (out = n * w + b), kind 1 = NormKind::Mod (out =
 * n * (1 + mods[scale * dim + j]) + mods[shift * dim + j]). mean and var
 * are sequential f32 sums divided by dim. */
void orc_layer_norm(const float *x, size_t rows, size_t dim, int kind, const float *w, const float *b,
                    const float *mods, size_t scale, size_t shift, float eps, float *out) {
    for (size_t r = 0; r < rows; r++) {
        const float *row = x + r * dim;
        float sum = 0.0f;
        for (size_t j = 0; j < dim; j++) sum += row[j];
        const float mean = sum / (float)dim;
        float vs = 0.0f;
        for (size_t j = 0; j < dim; j++) {
            const float c = row[j] - mean;
            vs += c * c;
        }
        const float var = vs / (float)dim;
        const float inv = 1.0f / sqrtf(var + eps);
        for (size_t j = 0; j < dim; j++) {
            const float n = (row[j] - mean) * inv;
            out[r * dim + j] = kind == 0 ? n * w[j] + b[j]
                                         : n * (1.0f + mods[scale * dim + j]) + mods[shift * dim + j];
        }
    }
}

/* CpuBackend::residual_norm, crates/lightx2v-cpu/src/lib.rs:364-392: in place
 * h += a * mods[gate] (gate < 0: h += a * 1.0), then normed = layer_norm(h). */
void orc_residual_norm(float *h, const float *a, size_t rows, size_t dim, const float *mods, long gate,
                       int kind, const float *w, const float *b, size_t scale, size_t shift, float eps,
                       float *normed) {
    for (size_t r = 0; r < rows; r++)
        for (size_t j = 0; j < dim; j++) {
            const float gv = gate >= 0 ? mods[(size_t)gate * dim + j] : 1.0f;
            h[r * dim + j] += a[r * dim + j] * gv;
        }
    orc_layer_norm(h, rows, dim, kind, w, b, mods, scale, shift, eps, normed);
}

/* CpuBackend::head_split, crates/lightx2v-cpu/src/lib.rs:406-459: columns
 * [col_off, col_off + heads * head_dim) of src (row stride src_stride) ->
 * out [heads, rows, head_dim]; with rms_w: x * (1 / sqrt(mean(x^2) + eps)) *
 * w[j] across all heads; with cos/sin ([rows, head_dim / 2]): interleaved
 * pairs (a, b) -> (a c - b s, a s + b c) within each head. */
void orc_head_split(const float *src, size_t rows, size_t src_stride, size_t col_off, size_t heads,
                    size_t head_dim, const float *rms_w, const float *cosv, const float *sinv, float eps,
                    float *out) {
    const size_t d = heads * head_dim;
    float *tmp = (float *)malloc(d * sizeof(float));
    for (size_t r = 0; r < rows; r++) {
        const float *row = src + r * src_stride + col_off;
        if (rms_w) {
            float ss = 0.0f;
            for (size_t j = 0; j < d; j++) ss += row[j] * row[j];
            const float ms = ss / (float)d;
            const float inv = 1.0f / sqrtf(ms + eps);
            for (size_t j = 0; j < d; j++) tmp[j] = row[j] * inv * rms_w[j];
        } else {
            memcpy(tmp, row, d * sizeof(float));
        }
        if (cosv && sinv) {
            for (size_t h = 0; h < heads; h++)
                for (size_t i = 0; i < head_dim / 2; i++) {
                    const float a = tmp[h * head_dim + 2 * i], bb = tmp[h * head_dim + 2 * i + 1];
                    const float c = cosv[r * head_dim / 2 + i], sn = sinv[r * head_dim / 2 + i];
                    tmp[h * head_dim + 2 * i] = a * c - bb * sn;
                    tmp[h * head_dim + 2 * i + 1] = a * sn + bb * c;
                }
        }
        for (size_t h = 0; h < heads; h++)
            for (size_t j = 0; j < head_dim; j++) out[(h * rows + r) * head_dim + j] = tmp[h * head_dim + j];
    }
    free(tmp);
}

int orc_openmp_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
