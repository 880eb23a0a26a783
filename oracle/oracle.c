/*
 * CPU oracle for decisive-b200.  TEST INFRASTRUCTURE ONLY -- never linked by the product.
 *
 * A plain-C restatement of the reference crate's quantised projection arithmetic
 * (decisive, src/models/pplx_flash/{int8,packed,quantization,quantized_rows,cpu,backbone}.rs).
 * Each function names the reference lines it follows.  Compiled with -ffp-contract=off so
 * that every `a * b + c` stays two roundings, exactly as Rust evaluates it; the places where
 * the reference fuses (the AVX2 `_mm256_fmadd_ps` of int8.rs:565) call fmaf explicitly.
 *
 * Parity pinning: the reference cannot be built here (Rust, no toolchain).  The restatement is
 * checked against the reference's own known-answer tests re-expressed in
 * tests/test_oracle_reference_vectors.py.
 */
#include "oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif
#if defined(__x86_64__)
#include <immintrin.h>
#endif

#define G ORACLE_GROUP

static inline float f32_of(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t bits_of(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float rust_max(float a, float b) { return a > b ? a : (isnan(a) ? b : (a < b ? b : a)); }
static inline float rust_min(float a, float b) { return a < b ? a : (isnan(a) ? b : (a > b ? b : a)); }
static inline float clampf(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }
/* f32::round_ties_even (default rounding mode is nearest-even) */
static inline float ties_even(float v) { return nearbyintf(v); }

/* ---------------------------------------------------------------- bf16 */
/* half 2.7.1 `bf16::from_f32`: round-to-nearest-even, NaN keeps its high bits and is quieted. */
uint16_t oracle_f32_to_bf16(float value) {
    uint32_t x = bits_of(value);
    if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x0040u);
    uint32_t round_bit = 0x00008000u;
    if ((x & round_bit) != 0 && (x & (3u * round_bit - 1u)) != 0) return (uint16_t)((x >> 16) + 1u);
    return (uint16_t)(x >> 16);
}
/* int8.rs:95-97: f32::from_bits((u16 as u32) << 16) */
float oracle_bf16_to_f32(uint16_t b) { return f32_of((uint32_t)b << 16); }
void oracle_f32_to_bf16_array(const float *x, size_t n, uint16_t *out) {
#pragma omp parallel for schedule(static) if (n > (1u << 16))
    for (size_t i = 0; i < n; ++i) out[i] = oracle_f32_to_bf16(x[i]);
}

/* ---------------------------------------------------------------- quantiser primitives */
/* int8.rs:305-313: (max |x| / limit).max(f32::MIN_POSITIVE); limit 7 for 4 bits else 127 */
float oracle_group_scale(const float *x, size_t n, int bits) {
    float limit = bits == 4 ? 7.f : 127.f;
    float m = 0.f;
    for (size_t i = 0; i < n; ++i) m = rust_max(m, fabsf(x[i]));
    return rust_max(m / limit, FLT_MIN);
}
/* int8.rs:347-360: (x * scale.recip()).round_ties_even().clamp(-limit, limit) */
void oracle_pack_codes(const float *x, size_t n, float scale, int bits, int8_t *out) {
    float limit = bits == 4 ? 7.f : 127.f;
    float inverse = 1.f / scale;
    for (size_t i = 0; i < n; ++i) out[i] = (int8_t)clampf(ties_even(x[i] * inverse), -limit, limit);
}

/* ---------------------------------------------------------------- packed rows (packed.rs) */
static size_t group_bytes(int bits) { return (size_t)G * bits / 8 + 4; }
/* packed.rs:10-19 */
size_t oracle_packed_size(size_t rows, size_t columns, int bits) {
    if (bits != 4 && bits != 8) return 0;
    if (rows == 0 || columns == 0 || columns % G) return 0;
    return rows * (columns / G) * group_bytes(bits);
}
/* packed.rs:22-28: Q4 nibble = code+8, low nibble first; Q8 two's complement */
static int packed_code(const uint8_t *group, size_t k, int bits) {
    if (bits == 4) return (int)((group[k / 2] >> (4 * (k % 2))) & 15) - 8;
    return (int)(int8_t)group[k];
}
/* packed.rs:31-56 */
int oracle_packed_pack(const uint16_t *bf16, size_t rows, size_t columns, int bits, uint8_t *out) {
    size_t total = oracle_packed_size(rows, columns, bits);
    if (!total) return -1;
    float limit = bits == 4 ? 7.f : 127.f;
    size_t groups = rows * columns / G, gb = group_bytes(bits);
    int bad = 0;
#pragma omp parallel for schedule(static) reduction(| : bad) if (groups > 4096)
    for (size_t gi = 0; gi < groups; ++gi) {
        float values[G];
        for (int i = 0; i < G; ++i) values[i] = oracle_bf16_to_f32(bf16[gi * G + i]);
        int finite = 1;
        for (int i = 0; i < G; ++i) finite &= isfinite(values[i]) ? 1 : 0;
        if (!finite) { bad |= 1; continue; }
        float m = 0.f;
        for (int i = 0; i < G; ++i) m = rust_max(m, fabsf(values[i]));
        float scale = rust_max(m / limit, FLT_MIN), inverse = 1.f / scale;
        uint8_t *o = out + gi * gb;
        if (bits == 4) {
            for (int i = 0; i < G; i += 2) {
                int a = (int)clampf(ties_even(values[i] * inverse), -limit, limit);
                int b = (int)clampf(ties_even(values[i + 1] * inverse), -limit, limit);
                o[i / 2] = (uint8_t)((a + 8) | ((b + 8) << 4));
            }
        } else {
            for (int i = 0; i < G; ++i) o[i] = (uint8_t)(int8_t)clampf(ties_even(values[i] * inverse), -limit, limit);
        }
        memcpy(o + gb - 4, &scale, 4);
    }
    return bad ? -2 : 0;
}
/* packed.rs:59-73: code as f32 * scale; scale must be finite and > 0 */
int oracle_packed_unpack(const uint8_t *packed, size_t bytes, int bits, float *out) {
    size_t stride = oracle_packed_size(1, G, bits);
    if (!stride || bytes == 0 || bytes % stride) return -1;
    size_t groups = bytes / stride;
    for (size_t gi = 0; gi < groups; ++gi) {
        const uint8_t *g = packed + gi * stride;
        float scale; memcpy(&scale, g + stride - 4, 4);
        if (!(isfinite(scale) && scale > 0.f)) return -1;
        for (int k = 0; k < G; ++k) out[gi * G + k] = (float)packed_code(g, k, bits) * scale;
    }
    return 0;
}
/* packed.rs:75-119: x quantised per 64 with /127, then sum += dot as f32 * (sx * sw) */
int oracle_packed_project(const uint8_t *packed, size_t bytes, int bits, size_t columns,
                          const float *x, size_t outputs, float *y) {
    size_t stride = oracle_packed_size(1, columns, bits);
    size_t gstride = oracle_packed_size(1, G, bits);
    if (!stride || bytes < outputs * stride) return -1;
    for (size_t i = 0; i < columns; ++i) if (!isfinite(x[i])) return -2;
    size_t groups = columns / G;
    int32_t *codes = (int32_t *)malloc(columns * sizeof(int32_t));
    float *scales = (float *)malloc(groups * sizeof(float));
    for (size_t g = 0; g < groups; ++g) {
        const float *v = x + g * G;
        float m = 0.f;
        for (int i = 0; i < G; ++i) m = rust_max(m, fabsf(v[i]));
        float s = rust_max(m / 127.f, FLT_MIN), inv = 1.f / s;
        for (int i = 0; i < G; ++i) codes[g * G + i] = (int32_t)clampf(ties_even(v[i] * inv), -127.f, 127.f);
        scales[g] = s;
    }
    for (size_t r = 0; r < outputs; ++r) {
        const uint8_t *row = packed + r * stride;
        float sum = 0.f;
        for (size_t g = 0; g < groups; ++g) {
            const uint8_t *grp = row + g * gstride;
            float s; memcpy(&s, grp + gstride - 4, 4);
            int32_t dot = 0;
            for (int k = 0; k < G; ++k) dot += codes[g * G + k] * packed_code(grp, k, bits);
            sum = sum + (float)dot * (scales[g] * s);
        }
        y[r] = sum;
    }
    free(codes); free(scales);
    return 0;
}

/* ---------------------------------------------------------------- fitted Q4 (quantization.rs) */
const float ORACLE_NF4[16] = {
    -1.f, -0.6961928f, -0.52507305f, -0.3949175f, -0.28444138f, -0.18477343f, -0.091050036f, 0.f,
    0.0795803f, 0.1609302f, 0.2461123f, 0.33791524f, 0.44070983f, 0.562617f, 0.72295684f, 1.f};

/* Rust `iter().sum::<f32>()` folds from -0.0 */
#define RUST_SUM_INIT (-0.0f)

/* quantization.rs:73-90 (scalar) and :92-128 (AVX2: 8 lanes, lane sums, then scalar tail) */
static void mse_stats(const float *x, size_t n, float scale, int simd, float out[3]) {
    float inverse = 1.f / scale;
    if (simd) {
        size_t end = n / 8 * 8;
        float num[8] = {0}, den[8] = {0}, err[8] = {0};
        for (size_t i = 0; i < end; i += 8)
            for (int j = 0; j < 8; ++j) {
                float v = x[i + j];
                float q = rust_min(7.f, rust_max(-8.f, ties_even(v * inverse)));
                float e = v - q * scale;
                num[j] = num[j] + v * q;
                den[j] = den[j] + q * q;
                err[j] = err[j] + e * e;
            }
        float tail[3];
        mse_stats(x + end, n - end, scale, 0, tail);
        float s0 = RUST_SUM_INIT, s1 = RUST_SUM_INIT, s2 = RUST_SUM_INIT;
        for (int j = 0; j < 8; ++j) { s0 = s0 + num[j]; s1 = s1 + den[j]; s2 = s2 + err[j]; }
        out[0] = s0 + tail[0]; out[1] = s1 + tail[1]; out[2] = s2 + tail[2];
        return;
    }
    float r0 = 0.f, r1 = 0.f, r2 = 0.f;
    for (size_t i = 0; i < n; ++i) {
        float v = x[i];
        float q = clampf(ties_even(v * inverse), -8.f, 7.f);
        float e = v - q * scale;
        r0 = r0 + v * q; r1 = r1 + q * q; r2 = r2 + e * e;
    }
    out[0] = r0; out[1] = r1; out[2] = r2;
}

/* quantization.rs:25-71 */
float oracle_fit_mse(const float *x, size_t n, int simd, int8_t *out) {
    float maximum = 0.f;
    for (size_t i = 0; i < n; ++i) maximum = rust_max(maximum, fabsf(x[i]));
    float baseline = oracle_group_scale(x, n, 4);
    oracle_pack_codes(x, n, baseline, 4, out);
    if (maximum == 0.f) return baseline;
    float values[G];
    for (size_t i = 0; i < n; ++i) values[i] = x[i] / maximum;
    float best_error = RUST_SUM_INIT;
    float ratio_b = baseline / maximum;
    for (size_t i = 0; i < n; ++i) {
        float e = values[i] - (float)out[i] * ratio_b;
        best_error = best_error + e * e;
    }
    float best = baseline;
    const float signs[2] = {-1.f, 1.f}, ratios[3] = {0.8f, 0.95f, 1.1f};
    for (int si = 0; si < 2; ++si)
        for (int ri = 0; ri < 3; ++ri) {
            float scale = signs[si] * ratios[ri] / 7.f;
            for (int it = 0; it < 4; ++it) {
                float st[3];
                mse_stats(values, n, scale, simd, st);
                if (st[2] < best_error) {
                    best_error = st[2];
                    best = scale * maximum;
                    float inv = 1.f / scale;
                    for (size_t i = 0; i < n; ++i) out[i] = (int8_t)clampf(ties_even(values[i] * inv), -8.f, 7.f);
                }
                if (st[1] == 0.f) break;
                float next = st[0] / st[1];
                if (!isfinite(next) || fabsf(next) < FLT_MIN || next == scale) break;
                scale = next;
            }
        }
    return best;
}

/* quantization.rs:202-258 */
static void affine_stats(const float *x, size_t n, float scale, float offset, int simd, float out[4]) {
    float inverse = 1.f / scale;
    if (simd) {
        size_t end = n / 8 * 8;
        float s[4][8];
        memset(s, 0, sizeof s);
        for (size_t i = 0; i < end; i += 8)
            for (int j = 0; j < 8; ++j) {
                float v = x[i + j];
                float q = rust_min(7.f, rust_max(-8.f, ties_even((v - offset) * inverse)));
                float e = v - (q * scale + offset);
                s[0][j] = s[0][j] + v * q;
                s[1][j] = s[1][j] + q * q;
                s[2][j] = s[2][j] + e * e;
                s[3][j] = s[3][j] + q;
            }
        float tail[4];
        affine_stats(x + end, n - end, scale, offset, 0, tail);
        for (int t = 0; t < 4; ++t) {
            float lanes = RUST_SUM_INIT;
            for (int j = 0; j < 8; ++j) lanes = lanes + s[t][j];
            out[t] = tail[t] + lanes;
        }
        return;
    }
    float a = 0.f, b = 0.f, c = 0.f, d = 0.f;
    for (size_t i = 0; i < n; ++i) {
        float v = x[i];
        float q = clampf(ties_even((v - offset) * inverse), -8.f, 7.f);
        float e = v - (q * scale + offset);
        a = a + v * q; b = b + q * q; c = c + e * e; d = d + q;
    }
    out[0] = a; out[1] = b; out[2] = c; out[3] = d;
}

/* quantization.rs:147-200 */
void oracle_fit_affine(const float *x, size_t n, int simd, int8_t *out, float *scale_out, float *offset_out) {
    float maximum = 0.f;
    for (size_t i = 0; i < n; ++i) maximum = rust_max(maximum, fabsf(x[i]));
    if (maximum == 0.f) {
        memset(out, 0, n);
        *scale_out = FLT_MIN; *offset_out = 0.f;
        return;
    }
    float values[G];
    for (size_t i = 0; i < n; ++i) values[i] = x[i] / maximum;
    float low = INFINITY, high = -INFINITY;
    for (size_t i = 0; i < n; ++i) { low = rust_min(low, values[i]); high = rust_max(high, values[i]); }
    if (low == high) {
        memset(out, 0, n);
        *scale_out = FLT_MIN; *offset_out = x[0];
        return;
    }
    float mean = RUST_SUM_INIT;
    for (size_t i = 0; i < n; ++i) mean = mean + values[i];
    mean = mean / (float)n;
    float best_error = INFINITY, best_s = 0.f, best_o = 0.f;
    const float ratios[3] = {0.8f, 1.f, 1.2f};
    for (int ri = 0; ri < 3; ++ri) {
        float scale = (high - low) / 15.f * ratios[ri];
        float offset = (high + low + scale) * 0.5f;
        for (int it = 0; it < 4; ++it) {
            float st[4];
            affine_stats(values, n, scale, offset, simd, st);
            if (st[2] < best_error) {
                best_error = st[2];
                best_s = scale * maximum;
                best_o = offset * maximum;
                float inv = 1.f / scale;
                for (size_t i = 0; i < n; ++i)
                    out[i] = (int8_t)clampf(ties_even((values[i] - offset) * inv), -8.f, 7.f);
            }
            float mean_q = st[3] / (float)n;
            float denominator = st[1] - st[3] * mean_q;
            if (denominator <= 0.f) break;
            float next = (st[0] - st[3] * mean) / denominator;
            if (!isfinite(next) || next <= 0.f) break;
            float next_offset = mean - next * mean_q;
            if (next == scale && next_offset == offset) break;
            scale = next; offset = next_offset;
        }
    }
    *scale_out = best_s; *offset_out = best_o;
}

/* quantization.rs:130-144 */
static int nf4_code(float value) {
    int low = 0, high = 15;
    while (low < high) {
        int middle = (low + high) / 2;
        if (value > (ORACLE_NF4[middle] + ORACLE_NF4[middle + 1]) * 0.5f) low = middle + 1;
        else high = middle;
    }
    return low;
}

/* quantization.rs:260-302 */
float oracle_fit_nf4(const float *x, size_t n, int8_t *out) {
    float maximum = 0.f;
    for (size_t i = 0; i < n; ++i) maximum = rust_max(maximum, fabsf(x[i]));
    if (maximum == 0.f) {
        memset(out, -1, n);
        return FLT_MIN;
    }
    float values[G];
    for (size_t i = 0; i < n; ++i) values[i] = x[i] / maximum;
    float best_error = INFINITY, best_scale = maximum;
    const float initials[3] = {0.85f, 1.f, 1.15f};
    for (int ii = 0; ii < 3; ++ii) {
        float scale = initials[ii];
        for (int it = 0; it < 4; ++it) {
            int8_t codes[G];
            memset(codes, 0, sizeof codes);
            float num = 0.f, den = 0.f, err = 0.f;
            for (size_t i = 0; i < n; ++i) {
                float v = values[i];
                int index = nf4_code(v / scale);
                codes[i] = (int8_t)(index - 8);
                float q = ORACLE_NF4[index];
                num = num + v * q;
                den = den + q * q;
                float d = v - scale * q;
                err = err + d * d;
            }
            if (err < best_error) {
                best_error = err;
                best_scale = scale * maximum;
                memcpy(out, codes, n);
            }
            if (den == 0.f) break;
            float next = num / den;
            if (next == scale || next <= 0.f) break;
            scale = next;
        }
    }
    return best_scale;
}

/* ---------------------------------------------------------------- int8::Matrix (int8.rs) */
size_t oracle_matrix_data_bytes(size_t input, size_t output, int weight_bits) {
    size_t groups = (input + G - 1) / G;
    return (output + 7) / 8 * groups * G * 8 / (weight_bits == 4 ? 2 : 1);
}
size_t oracle_matrix_scale_count(size_t input, size_t output) {
    return (output + 7) / 8 * ((input + G - 1) / G) * 8;
}

/* int8.rs:51-152 (panel layout :121-132) */
int oracle_matrix_from_bf16(const uint16_t *bf16, size_t input, size_t output, int weight_bits,
                            int fit, int simd, int8_t *data, float *scales, float *offsets) {
    if (weight_bits != 4 && weight_bits != 8) return -1;
    if (input == 0 || output == 0) return -1;
    if (fit == 2 && weight_bits != 4) return -1;
    size_t groups = (input + G - 1) / G;
    size_t panels = (output + 7) / 8;
    size_t panel_bytes = groups * G * 8 / (weight_bits == 4 ? 2 : 1);
    memset(data, 0, panels * panel_bytes);
    memset(scales, 0, panels * groups * 8 * sizeof(float));
    if (offsets) memset(offsets, 0, panels * groups * 8 * sizeof(float));
    int bad = 0;
#pragma omp parallel for schedule(dynamic, 4) reduction(| : bad)
    for (size_t panel = 0; panel < panels; ++panel) {
        int8_t *pd = data + panel * panel_bytes;
        float *ps = scales + panel * groups * 8;
        float *po = offsets ? offsets + panel * groups * 8 : NULL;
        size_t cmax = output - panel * 8 < 8 ? output - panel * 8 : 8;
        for (size_t c = 0; c < cmax; ++c)
            for (size_t g = 0; g < groups; ++g) {
                size_t count = input - g * G < G ? input - g * G : G;
                float values[G];
                memset(values, 0, sizeof values);
                for (size_t k = 0; k < count; ++k)
                    values[k] = oracle_bf16_to_f32(bf16[(panel * 8 + c) * input + g * G + k]);
                int finite = 1;
                for (int k = 0; k < G; ++k) finite &= isfinite(values[k]) ? 1 : 0;
                if (!finite) { bad |= 1; continue; }
                int8_t codes[G];
                memset(codes, 0, sizeof codes);
                float s;
                if (fit == 2) {
                    float b;
                    oracle_fit_affine(values, count, simd, codes, &s, &b);
                    if (po) po[g * 8 + c] = b;
                } else if (fit == 1 && weight_bits == 4) {
                    s = oracle_fit_mse(values, count, simd, codes);
                } else {
                    s = oracle_group_scale(values, G, weight_bits);
                    oracle_pack_codes(values, G, s, weight_bits, codes);
                }
                ps[g * 8 + c] = s;
                for (int k = 0; k < G; k += 4) {
                    size_t at = g * G * 8 + (size_t)k / 4 * 32 + c * 4;
                    if (weight_bits == 4) {
                        for (int j = 0; j < 2; ++j)
                            pd[at / 2 + j] = (int8_t)(uint8_t)((codes[k + 2 * j] + 8) | ((codes[k + 2 * j + 1] + 8) << 4));
                    } else {
                        memcpy(pd + at, codes + k, 4);
                    }
                }
            }
    }
    return bad ? -2 : 0;
}

/* int8.rs:178-202 */
void oracle_matrix_prepare(const float *x, size_t tokens, size_t input, int activation_bits,
                           int8_t *values, float *scales, int32_t *sums) {
    size_t groups = (input + G - 1) / G;
#pragma omp parallel for schedule(static) if (tokens > 8)
    for (size_t r = 0; r < tokens; ++r) {
        const float *row = x + r * input;
        for (size_t g = 0; g < groups; ++g) {
            size_t count = input - g * G < G ? input - g * G : G;
            float s = oracle_group_scale(row + g * G, count, activation_bits);
            scales[r * groups + g] = s;
            int8_t *out = values + (r * groups + g) * G;
            memset(out, 0, G);
            oracle_pack_codes(row + g * G, count, s, activation_bits, out);
            if (sums) {
                int32_t t = 0;
                for (int k = 0; k < G; ++k) t += out[k];
                sums[r * groups + g] = t;
            }
        }
    }
}

/* panel index of weight (c, g, k), int8.rs:270-273 */
static inline int weight_code(const int8_t *data, int weight_bits, size_t groups, size_t c, size_t g, size_t k) {
    size_t index = (c / 8 * groups + g) * G * 8 + k / 4 * 32 + c % 8 * 4 + k % 4;
    if (weight_bits == 4) return (int)(((uint8_t)data[index / 2] >> (index % 2 * 4)) & 15) - 8;
    return data[index];
}

/* modes 0 and 1: scalar restatements of int8.rs:526-585 (fma) and int8.rs:259-287 (mul+add) */
static void apply_scalar(const int8_t *data, const float *scales, const float *offsets, size_t input,
                         size_t output, int weight_bits, const int8_t *values, const float *act_scales,
                         const int32_t *sums, size_t tokens, int fused, float *y) {
    size_t groups = (input + G - 1) / G;
#pragma omp parallel for schedule(dynamic, 1)
    for (size_t c = 0; c < output; ++c) {
        int8_t w[G];
        for (size_t r = 0; r < tokens; ++r) y[r * output + c] = 0.f;
        float *acc = (float *)calloc(tokens, sizeof(float));
        for (size_t g = 0; g < groups; ++g) {
            for (int k = 0; k < G; ++k) w[k] = (int8_t)weight_code(data, weight_bits, groups, c, g, k);
            size_t si = (c / 8 * groups + g) * 8 + c % 8;
            float sw = scales[si];
            for (size_t r = 0; r < tokens; ++r) {
                const int8_t *a = values + (r * groups + g) * G;
                int32_t dot = 0;
                for (int k = 0; k < G; ++k) dot += (int32_t)a[k] * (int32_t)w[k];
                float sa = act_scales[r * groups + g];
                if (fused) {
                    acc[r] = fmaf((float)dot, sw * sa, acc[r]);
                    if (offsets) acc[r] = fmaf(offsets[si], sa * (float)sums[r * groups + g], acc[r]);
                } else {
                    acc[r] = acc[r] + (float)dot * (sa * sw);
                    if (offsets) acc[r] = acc[r] + offsets[si] * (sa * (float)sums[r * groups + g]);
                }
            }
        }
        for (size_t r = 0; r < tokens; ++r) y[r * output + c] = acc[r];
        free(acc);
    }
}

#if defined(__x86_64__)
/* int8.rs:484-492: 16 packed bytes -> 32 signed codes, natural order */
__attribute__((target("avx2,fma"))) static inline __m256i unpack_q4(const int8_t *d) {
    __m256i packed = _mm256_cvtepu8_epi16(_mm_loadu_si128((const __m128i *)d));
    __m256i low = _mm256_and_si256(packed, _mm256_set1_epi16(0x000f));
    __m256i high = _mm256_and_si256(_mm256_slli_epi16(packed, 4), _mm256_set1_epi16(0x0f00));
    return _mm256_sub_epi8(_mm256_or_si256(low, high), _mm256_set1_epi8(8));
}

/* int8.rs:526-585 rows<R,Q4>, with R a runtime count <= 7 */
__attribute__((target("avx2,fma"))) static void rows_avx2(size_t R, int q4, size_t groups, size_t output,
                                                         const int8_t *values, const float *act_scales,
                                                         const int32_t *sums, const float *offsets,
                                                         float *out, size_t first, size_t panel,
                                                         const int8_t *pdata, const float *pscales) {
    const __m256i one = _mm256_set1_epi16(1);
    __m256 acc_sum[7];
    for (size_t r = 0; r < R; ++r) acc_sum[r] = _mm256_setzero_ps();
    for (size_t g = 0; g < groups; ++g) {
        __m256i acc[7];
        for (size_t r = 0; r < R; ++r) acc[r] = _mm256_setzero_si256();
        size_t base = g * G * 8;
        for (size_t k = 0; k < G; k += 4) {
            __m256i b = q4 ? unpack_q4(pdata + (base + k * 8) / 2)
                           : _mm256_loadu_si256((const __m256i *)(pdata + base + k * 8));
            __m256i magnitude = _mm256_abs_epi8(b);
            for (size_t r = 0; r < R; ++r) {
                int32_t word;
                memcpy(&word, values + ((first + r) * groups + g) * G + k, 4);
                __m256i a = _mm256_set1_epi32(word);
                __m256i pair = _mm256_maddubs_epi16(magnitude, _mm256_sign_epi8(a, b));
                acc[r] = _mm256_add_epi32(acc[r], _mm256_madd_epi16(pair, one));
            }
        }
        __m256 sw = _mm256_loadu_ps(pscales + g * 8);
        for (size_t r = 0; r < R; ++r) {
            float sa = act_scales[(first + r) * groups + g];
            __m256 s = _mm256_mul_ps(sw, _mm256_set1_ps(sa));
            acc_sum[r] = _mm256_fmadd_ps(_mm256_cvtepi32_ps(acc[r]), s, acc_sum[r]);
            if (offsets) {
                __m256 off = _mm256_loadu_ps(offsets + (panel * groups + g) * 8);
                float sx = sa * (float)sums[(first + r) * groups + g];
                acc_sum[r] = _mm256_fmadd_ps(off, _mm256_set1_ps(sx), acc_sum[r]);
            }
        }
    }
    for (size_t r = 0; r < R; ++r) {
        float *dst = out + (first + r) * output + panel * 8;
        if (panel * 8 + 8 <= output) {
            _mm256_storeu_ps(dst, acc_sum[r]);
        } else {
            float tail[8];
            _mm256_storeu_ps(tail, acc_sum[r]);
            memcpy(dst, tail, (output - panel * 8) * sizeof(float));
        }
    }
}

/* int8.rs:229-258 + project_buffered :448-480 + project_panel :496-522 */
__attribute__((target("avx2,fma"))) static void apply_avx2(const int8_t *data, const float *scales,
                                                          const float *offsets, size_t input, size_t output,
                                                          int weight_bits, const int8_t *values,
                                                          const float *act_scales, const int32_t *sums,
                                                          size_t tokens, float *y) {
    size_t groups = (input + G - 1) / G;
    size_t panels = (output + 7) / 8;
    size_t tiles = (output + 31) / 32;
    size_t count = groups * G * 8;
    int q4 = weight_bits == 4;
#pragma omp parallel
    {
        int8_t *expanded = (int8_t *)aligned_alloc(64, (count + 63) / 64 * 64);
#pragma omp for schedule(dynamic, 1)
        for (size_t tile = 0; tile < tiles; ++tile) {
            size_t start = tile * 4, end = start + 4 < panels ? start + 4 : panels;
            for (size_t panel = start; panel < end; ++panel) {
                const int8_t *pd = data + panel * count / (q4 ? 2 : 1);
                const float *ps = scales + panel * groups * 8;
                int packed = q4;
                if (q4 && tokens >= 16) {
                    for (size_t at = 0; at < count; at += 32)
                        _mm256_storeu_si256((__m256i *)(expanded + at), unpack_q4(pd + at / 2));
                    pd = expanded;
                    packed = 0;
                }
                size_t full = tokens / 4 * 4;
                for (size_t r = 0; r < full; r += 4)
                    rows_avx2(4, packed, groups, output, values, act_scales, sums, offsets, y, r, panel, pd, ps);
                if (tokens > full)
                    rows_avx2(tokens - full, packed, groups, output, values, act_scales, sums, offsets, y, full,
                              panel, pd, ps);
            }
        }
        free(expanded);
    }
}
#endif

int oracle_has_avx2(void) {
#if defined(__x86_64__)
    __builtin_cpu_init();
    return __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
#else
    return 0;
#endif
}

void oracle_matrix_apply_prepared(const int8_t *data, const float *scales, const float *offsets,
                                  size_t input, size_t output, int weight_bits,
                                  const int8_t *values, const float *act_scales,
                                  const int32_t *sums, size_t tokens, int mode, float *y) {
    if (tokens == 0) return;
#if defined(__x86_64__)
    if (mode == 2 && oracle_has_avx2()) {
        apply_avx2(data, scales, offsets, input, output, weight_bits, values, act_scales, sums, tokens, y);
        return;
    }
#endif
    apply_scalar(data, scales, offsets, input, output, weight_bits, values, act_scales, sums, tokens,
                 mode != 1, y);
}

/* int8.rs:166-176: non-finite input -> every output NaN */
void oracle_matrix_apply(const int8_t *data, const float *scales, const float *offsets,
                         size_t input, size_t output, int weight_bits, int activation_bits,
                         const float *x, size_t tokens, int mode, float *y) {
    size_t n = tokens * input;
    for (size_t i = 0; i < n; ++i)
        if (!isfinite(x[i])) {
            for (size_t j = 0; j < tokens * output; ++j) y[j] = NAN;
            return;
        }
    size_t groups = (input + G - 1) / G;
    int8_t *values = (int8_t *)malloc(tokens * groups * G + 1);
    float *sc = (float *)malloc((tokens * groups + 1) * sizeof(float));
    int32_t *sums = offsets ? (int32_t *)malloc((tokens * groups + 1) * sizeof(int32_t)) : NULL;
    oracle_matrix_prepare(x, tokens, input, activation_bits, values, sc, sums);
    oracle_matrix_apply_prepared(data, scales, offsets, input, output, weight_bits, values, sc, sums, tokens,
                                 mode, y);
    free(values); free(sc); free(sums);
}

/* ---------------------------------------------------------------- embedding rows */
/* quantized_rows.rs:21-87 */
int oracle_embedding_from_bf16(const uint16_t *bf16, size_t rows, size_t columns, int bits,
                               int fit, int simd, uint8_t *data, float *scales, float *offsets) {
    if ((bits != 4 && bits != 8) || columns == 0 || columns % G) return -1;
    if (fit == 3 && bits != 4) return -1;
    if (fit == 2 && bits != 4) return -1;
    size_t groups = rows * columns / G, stride = (size_t)G * bits / 8;
    int bad = 0;
#pragma omp parallel for schedule(static) reduction(| : bad) if (groups > 4096)
    for (size_t gi = 0; gi < groups; ++gi) {
        float values[G];
        for (int i = 0; i < G; ++i) values[i] = oracle_bf16_to_f32(bf16[gi * G + i]);
        int finite = 1;
        for (int i = 0; i < G; ++i) finite &= isfinite(values[i]) ? 1 : 0;
        if (!finite) { bad |= 1; continue; }
        int8_t codes[G];
        memset(codes, 0, sizeof codes);
        float s, b = 0.f;
        if (fit == 2) oracle_fit_affine(values, G, simd, codes, &s, &b);
        else if (fit == 3) s = oracle_fit_nf4(values, G, codes);
        else if (fit == 1 && bits == 4) s = oracle_fit_mse(values, G, simd, codes);
        else {
            s = oracle_group_scale(values, G, bits);
            oracle_pack_codes(values, G, s, bits, codes);
        }
        scales[gi] = s;
        if (offsets) offsets[gi] = b;
        uint8_t *o = data + gi * stride;
        for (size_t i = 0; i < stride; ++i)
            o[i] = bits == 4 ? (uint8_t)((codes[2 * i] + 8) | ((codes[2 * i + 1] + 8) << 4)) : (uint8_t)codes[i];
    }
    return bad ? -2 : 0;
}
/* quantized_rows.rs:89-110 */
void oracle_embedding_append(const uint8_t *data, const float *scales, const float *offsets,
                             size_t columns, int bits, int nf4, size_t id, float *out) {
    size_t first = id * columns;
    for (size_t i = 0; i < columns; ++i) {
        size_t at = first + i;
        int code = bits == 4 ? (int)((data[at / 2] >> (at % 2 * 4)) & 15) - 8 : (int)(int8_t)data[at];
        float vc = nf4 ? ORACLE_NF4[code + 8] : (float)code;
        float v = vc * scales[at / G];
        if (offsets) v = v + offsets[at / G];
        out[i] = v;
    }
}

/* ---------------------------------------------------------------- layer math */
/* cpu.rs:310-333 (rms_from): scale = 1 / sqrt(sum(v*v)/n + eps); out = (v*scale) * w or (1+w) */
void oracle_rms(const float *x, float *y, size_t rows, size_t width, const float *weight, float eps,
                int zero_centered) {
#pragma omp parallel for schedule(static) if (rows > 16)
    for (size_t r = 0; r < rows; ++r) {
        const float *src = x + r * width;
        float sum = RUST_SUM_INIT;
        for (size_t i = 0; i < width; ++i) sum = sum + src[i] * src[i];
        float scale = 1.f / sqrtf(sum / (float)width + eps);
        for (size_t i = 0; i < width; ++i)
            y[r * width + i] = (src[i] * scale) * (zero_centered ? 1.f + weight[i] : weight[i]);
    }
}
/* cpu.rs:513-518 */
static inline float sigmoid(float x) { return 1.f / (1.f + expf(-x)); }
static inline float silu(float x) { return x * sigmoid(x); }
/* cpu.rs:348-371 (portable branch) */
void oracle_silu_mul(float *gate, const float *up, size_t n) {
#pragma omp parallel for schedule(static) if (n > 65536)
    for (size_t i = 0; i < n; ++i) gate[i] = silu(gate[i]) * up[i];
}
/* cpu.rs:519-529 */
void oracle_softmax(float *x, size_t n) {
    float m = -INFINITY;
    for (size_t i = 0; i < n; ++i) m = rust_max(m, x[i]);
    float sum = 0.f;
    for (size_t i = 0; i < n; ++i) { x[i] = expf(x[i] - m); sum = sum + x[i]; }
    for (size_t i = 0; i < n; ++i) x[i] = x[i] / sum;
}
/* backbone.rs:471-483 rotate-half over the first `rotary` dims of each head;
 * inv_freq[i] = 1 / theta^(2i/rotary) (backbone.rs:214-216) */
void oracle_rope(float *x, size_t tokens, size_t heads, size_t head_dim, size_t rotary, size_t offset,
                 float theta) {
    size_t half = rotary / 2;
    float *freq = (float *)malloc(half * sizeof(float));
    for (size_t i = 0; i < half; ++i) freq[i] = 1.f / powf(theta, (float)(2 * i) / (float)rotary);
#pragma omp parallel for schedule(static) if (tokens > 16)
    for (size_t t = 0; t < tokens; ++t)
        for (size_t h = 0; h < heads; ++h) {
            float *head = x + (t * heads + h) * head_dim;
            for (size_t i = 0; i < half; ++i) {
                float angle = (float)(offset + t) * freq[i];
                float c = cosf(angle), s = sinf(angle);
                float a = head[i], b = head[i + half];
                head[i] = a * c - b * s;
                head[i + half] = b * c + a * s;
            }
        }
    free(freq);
}
/* backbone.rs:560-600: per head, scores = scale * q k^T, softmax, P v (non-causal) */
void oracle_attention(const float *q, const float *k, const float *v, size_t tokens, size_t q_heads,
                      size_t kv_heads, size_t head_dim, float scale, float *out) {
    oracle_attention_masked(q, k, v, tokens, q_heads, kv_heads, head_dim, scale, 0, out);
}

void oracle_attention_masked(const float *q, const float *k, const float *v, size_t tokens, size_t q_heads,
                             size_t kv_heads, size_t head_dim, float scale, int causal, float *out) {
    size_t per = q_heads / kv_heads;
#pragma omp parallel
    {
        float *scores = (float *)malloc(tokens * sizeof(float));
        float *acc = (float *)malloc(head_dim * sizeof(float));
#pragma omp for collapse(2) schedule(dynamic, 8)
        for (size_t h = 0; h < q_heads; ++h)
            for (size_t i = 0; i < tokens; ++i) {
                size_t kh = h / per;
                const size_t keys = causal ? i + 1 : tokens;
                const float *qi = q + (i * q_heads + h) * head_dim;
                for (size_t j = 0; j < keys; ++j) {
                    const float *kj = k + (j * kv_heads + kh) * head_dim;
                    float dot = 0.f;
                    for (size_t d = 0; d < head_dim; ++d) dot = fmaf(qi[d], kj[d], dot);
                    scores[j] = scale * dot;
                }
                oracle_softmax(scores, keys);
                for (size_t d = 0; d < head_dim; ++d) acc[d] = 0.f;
                for (size_t j = 0; j < keys; ++j) {
                    const float *vj = v + (j * kv_heads + kh) * head_dim;
                    for (size_t d = 0; d < head_dim; ++d) acc[d] = fmaf(scores[j], vj[d], acc[d]);
                }
                memcpy(out + (i * q_heads + h) * head_dim, acc, head_dim * sizeof(float));
            }
        free(scores); free(acc);
    }
}

/* ---------------------------------------------------------------- composed encoder */
typedef struct {
    int8_t *data;
    float *scales;
    size_t input, output;
} qmatrix;

typedef struct {
    oracle_encoder_config cfg;
    uint8_t *emb_data;
    float *emb_scales;
    qmatrix *q, *k, *v, *o, *gate, *up, *down;
    float **input_norm, **post_norm, **q_norm, **k_norm;
    float *final_norm;
} encoder;

static int qmatrix_init(qmatrix *m, const uint16_t *w, size_t input, size_t output, int bits) {
    m->input = input; m->output = output;
    m->data = (int8_t *)malloc(oracle_matrix_data_bytes(input, output, bits));
    m->scales = (float *)malloc(oracle_matrix_scale_count(input, output) * sizeof(float));
    return oracle_matrix_from_bf16(w, input, output, bits, 0, 1, m->data, m->scales, NULL);
}
static void qmatrix_free(qmatrix *m) { free(m->data); free(m->scales); }

static float *copy_floats(const float *x, size_t n) {
    float *y = (float *)malloc(n * sizeof(float));
    memcpy(y, x, n * sizeof(float));
    return y;
}

void *oracle_encoder_create(const oracle_encoder_config *cfg, const oracle_encoder_weights *w) {
    encoder *e = (encoder *)calloc(1, sizeof(encoder));
    e->cfg = *cfg;
    size_t L = cfg->layers, D = cfg->hidden, Hq = cfg->q_heads, Hk = cfg->kv_heads, Dh = cfg->head_dim,
           F = cfg->ffn, V = cfg->vocab;
    int bits = cfg->weight_bits;
    e->emb_data = (uint8_t *)malloc(V * D * bits / 8);
    e->emb_scales = (float *)malloc(V * D / G * sizeof(float));
    int rc = oracle_embedding_from_bf16(w->embedding, V, D, bits, 0, 1, e->emb_data, e->emb_scales, NULL);
    e->q = calloc(L, sizeof(qmatrix)); e->k = calloc(L, sizeof(qmatrix)); e->v = calloc(L, sizeof(qmatrix));
    e->o = calloc(L, sizeof(qmatrix)); e->gate = calloc(L, sizeof(qmatrix)); e->up = calloc(L, sizeof(qmatrix));
    e->down = calloc(L, sizeof(qmatrix));
    e->input_norm = calloc(L, sizeof(float *)); e->post_norm = calloc(L, sizeof(float *));
    e->q_norm = calloc(L, sizeof(float *)); e->k_norm = calloc(L, sizeof(float *));
    for (size_t l = 0; l < L && rc == 0; ++l) {
        rc |= qmatrix_init(&e->q[l], w->q[l], D, Hq * Dh, bits);
        rc |= qmatrix_init(&e->k[l], w->k[l], D, Hk * Dh, bits);
        rc |= qmatrix_init(&e->v[l], w->v[l], D, Hk * Dh, bits);
        rc |= qmatrix_init(&e->o[l], w->o[l], Hq * Dh, D, bits);
        rc |= qmatrix_init(&e->gate[l], w->gate[l], D, F, bits);
        rc |= qmatrix_init(&e->up[l], w->up[l], D, F, bits);
        rc |= qmatrix_init(&e->down[l], w->down[l], F, D, bits);
        e->input_norm[l] = copy_floats(w->input_norm[l], D);
        e->post_norm[l] = copy_floats(w->post_norm[l], D);
        e->q_norm[l] = copy_floats(w->q_norm[l], Dh);
        e->k_norm[l] = copy_floats(w->k_norm[l], Dh);
    }
    e->final_norm = copy_floats(w->final_norm, D);
    if (rc) { oracle_encoder_destroy(e); return NULL; }
    return e;
}

void oracle_encoder_destroy(void *p) {
    encoder *e = (encoder *)p;
    if (!e) return;
    for (int l = 0; l < e->cfg.layers; ++l) {
        if (e->q) qmatrix_free(&e->q[l]);
        if (e->k) qmatrix_free(&e->k[l]);
        if (e->v) qmatrix_free(&e->v[l]);
        if (e->o) qmatrix_free(&e->o[l]);
        if (e->gate) qmatrix_free(&e->gate[l]);
        if (e->up) qmatrix_free(&e->up[l]);
        if (e->down) qmatrix_free(&e->down[l]);
        if (e->input_norm) free(e->input_norm[l]);
        if (e->post_norm) free(e->post_norm[l]);
        if (e->q_norm) free(e->q_norm[l]);
        if (e->k_norm) free(e->k_norm[l]);
    }
    free(e->q); free(e->k); free(e->v); free(e->o); free(e->gate); free(e->up); free(e->down);
    free(e->input_norm); free(e->post_norm); free(e->q_norm); free(e->k_norm);
    free(e->final_norm); free(e->emb_data); free(e->emb_scales);
    free(e);
}

static void project(const qmatrix *m, int bits, int abits, const float *x, size_t tokens, int mode, float *y) {
    oracle_matrix_apply(m->data, m->scales, NULL, m->input, m->output, bits, abits, x, tokens, mode, y);
}

/* Pre-norm residual block (backbone.rs:197-249) with a Qwen3 attention mixer:
 * x += o(attn(rope(qnorm(q(n))), rope(knorm(k(n))), v(n))), n = rms(x);
 * x += down(silu(gate(n)) * up(n)), n = rms(x). */
int oracle_encoder_forward(void *p, const int32_t *ids, size_t T, int layers_limit, int mode, float *pooled,
                           float *hidden_out) {
    encoder *e = (encoder *)p;
    const oracle_encoder_config *c = &e->cfg;
    size_t D = c->hidden, Hq = c->q_heads, Hk = c->kv_heads, Dh = c->head_dim, F = c->ffn;
    int bits = c->weight_bits, abits = c->activation_bits;
    int L = layers_limit < 0 || layers_limit > c->layers ? c->layers : layers_limit;
    for (size_t t = 0; t < T; ++t)
        if (ids[t] < 0 || ids[t] >= c->vocab) return -1;
    float *x = malloc(T * D * sizeof(float)), *n = malloc(T * D * sizeof(float));
    float *q = malloc(T * Hq * Dh * sizeof(float)), *k = malloc(T * Hk * Dh * sizeof(float));
    float *v = malloc(T * Hk * Dh * sizeof(float)), *ctx = malloc(T * Hq * Dh * sizeof(float));
    float *proj = malloc(T * D * sizeof(float));
    float *g = malloc(T * F * sizeof(float)), *u = malloc(T * F * sizeof(float));
    for (size_t t = 0; t < T; ++t)
        oracle_embedding_append(e->emb_data, e->emb_scales, NULL, D, bits, 0, (size_t)ids[t], x + t * D);
    float scale = 1.f / sqrtf((float)Dh);
    for (int l = 0; l < L; ++l) {
        oracle_rms(x, n, T, D, e->input_norm[l], c->eps, 0);
        project(&e->q[l], bits, abits, n, T, mode, q);
        project(&e->k[l], bits, abits, n, T, mode, k);
        project(&e->v[l], bits, abits, n, T, mode, v);
        oracle_rms(q, q, T * Hq, Dh, e->q_norm[l], c->eps, 0);
        oracle_rms(k, k, T * Hk, Dh, e->k_norm[l], c->eps, 0);
        oracle_rope(q, T, Hq, Dh, Dh, 0, c->rope_theta);
        oracle_rope(k, T, Hk, Dh, Dh, 0, c->rope_theta);
        oracle_attention_masked(q, k, v, T, Hq, Hk, Dh, scale, e->cfg.causal, ctx);
        project(&e->o[l], bits, abits, ctx, T, mode, proj);
        for (size_t i = 0; i < T * D; ++i) x[i] = x[i] + proj[i];
        oracle_rms(x, n, T, D, e->post_norm[l], c->eps, 0);
        project(&e->gate[l], bits, abits, n, T, mode, g);
        project(&e->up[l], bits, abits, n, T, mode, u);
        oracle_silu_mul(g, u, T * F);
        project(&e->down[l], bits, abits, g, T, mode, proj);
        for (size_t i = 0; i < T * D; ++i) x[i] = x[i] + proj[i];
    }
    oracle_rms(x, n, T, D, e->final_norm, c->eps, 0);
    if (hidden_out) memcpy(hidden_out, n, T * D * sizeof(float));
    for (size_t d = 0; d < D; ++d) {
        float s = 0.f;
        for (size_t t = 0; t < T; ++t) s = s + n[t * D + d];
        pooled[d] = s / (float)T;
    }
    free(x); free(n); free(q); free(k); free(v); free(ctx); free(proj); free(g); free(u);
    return 0;
}

/* ---------------------------------------------------------------- Decima int8 */

/* decima/int8.rs:413-415: (max over |x| starting at 0) / 127, at least f32::MIN_POSITIVE. */
float oracle_decima_scale(const float *x, size_t n) {
    float m = 0.f;
    for (size_t i = 0; i < n; ++i) {
        const float a = fabsf(x[i]);
        m = a > m ? a : m;  /* Rust f32::max; inputs are finite here */
    }
    const float s = m / 127.f;
    return s > FLT_MIN ? s : FLT_MIN;
}

/* decima/int8.rs:416-418: (x / s).round() -- half away from zero -- clamped to [-127, 127]. */
int8_t oracle_decima_quantize(float x, float scale) {
    float q = roundf(x / scale);
    if (q < -127.f) q = -127.f;
    if (q > 127.f) q = 127.f;
    return (int8_t)q;
}

/* decima/int8.rs:106-151 (Matrix::new) and :239-253 (the activation fill): each row in blocks,
 * the last block partial; codes past cols stay 0. */
void oracle_decima_quantize_rows(const float *x, size_t rows, size_t cols, size_t block, int8_t *codes,
                                 float *scales) {
    const size_t groups = (cols + block - 1) / block;
    for (size_t r = 0; r < rows; ++r) {
        int8_t *row = codes + r * groups * block;
        memset(row, 0, groups * block);
        for (size_t g = 0; g < groups; ++g) {
            const size_t s0 = g * block, len = (s0 + block < cols ? s0 + block : cols) - s0;
            const float *v = x + r * cols + s0;
            const float sc = oracle_decima_scale(v, len);
            scales[r * groups + g] = sc;
            for (size_t k = 0; k < len; ++k) row[s0 + k] = oracle_decima_quantize(v[k], sc);
        }
    }
}

void oracle_decima_apply_w8a8(const int8_t *w_codes, const float *w_scales, size_t rows, size_t cols,
                              size_t block, const float *x, size_t m, const float *bias, int mode, float *y) {
    const size_t groups = (cols + block - 1) / block;
    for (size_t i = 0; i < m * cols; ++i)
        if (!isfinite(x[i])) {
            for (size_t j = 0; j < m * rows; ++j) y[j] = NAN;
            return;
        }
    int8_t *a = malloc(m * groups * block);
    float *sa = malloc(m * groups * sizeof(float));
    oracle_decima_quantize_rows(x, m, cols, block, a, sa);
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)m; ++i) {
        for (size_t n = 0; n < rows; ++n) {
            float sum = 0.f;
            for (size_t g = 0; g < groups; ++g) {
                const int8_t *qa = a + ((size_t)i * groups + g) * block;
                const int8_t *qw = w_codes + (n * groups + g) * block;
                int32_t dot = 0;
                for (size_t k = 0; k < block; ++k) dot += (int32_t)qa[k] * (int32_t)qw[k];
                const float s = w_scales[n * groups + g] * sa[(size_t)i * groups + g];
                if (mode == 0) sum = fmaf((float)dot, s, sum);
                else sum = sum + (float)dot * s;
            }
            y[(size_t)i * rows + n] = sum + (bias ? bias[n] : 0.f);
        }
    }
    free(a);
    free(sa);
}

/* Matrix::apply_with_rows in Weights mode (W8A32: int8 weights, f32 activations).
 * mode 0, the AVX2 kernel (decima/int8/weights_x86.rs:51-113): every weight is decoded to the f32
 *   product code * scale (:63-76), then each output is one fma chain over k = 0..cols-1 from 0
 *   (:86-100), plus the bias (:104-109);
 * mode 1, the portable kernel (decima/int8.rs:384-407): per block a dot of x * code (a multiply
 *   and an add per term), then sum += dot * scale, then the bias.
 * A non-finite x gives all-NaN y (int8.rs:183-187).  codes [rows, groups*block], scales
 * [rows, groups]. */
void oracle_decima_apply_w8a32(const int8_t *w_codes, const float *w_scales, size_t rows, size_t cols,
                               size_t block, const float *x, size_t m, const float *bias, int mode, float *y) {
    const size_t groups = (cols + block - 1) / block;
    for (size_t i = 0; i < m * cols; ++i)
        if (!isfinite(x[i])) {
            for (size_t j = 0; j < m * rows; ++j) y[j] = NAN;
            return;
        }
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)m; ++i) {
        const float *xi = x + (size_t)i * cols;
        for (size_t n = 0; n < rows; ++n) {
            const int8_t *qw = w_codes + n * groups * block;
            float sum = 0.f;
            if (mode == 0) {
                for (size_t k = 0; k < cols; ++k) {
                    const float wf = (float)qw[k] * w_scales[n * groups + k / block];
                    sum = fmaf(xi[k], wf, sum);
                }
            } else {
                for (size_t g = 0; g < groups; ++g) {
                    float dot = 0.f;
                    const size_t k1 = (g + 1) * block < cols ? (g + 1) * block : cols;
                    for (size_t k = g * block; k < k1; ++k) dot = dot + xi[k] * (float)qw[k];
                    sum = sum + dot * w_scales[n * groups + g];
                }
            }
            y[(size_t)i * rows + n] = sum + (bias ? bias[n] : 0.f);
        }
    }
}

void oracle_layer_norm(float *x, size_t rows, size_t d, const float *w, const float *b, float eps) {
    for (size_t r = 0; r < rows; ++r) {
        float *row = x + r * d;
        float sum = 0.f;
        for (size_t i = 0; i < d; ++i) sum += row[i];
        const float mean = sum / (float)d;
        float var = 0.f;
        for (size_t i = 0; i < d; ++i) var += (row[i] - mean) * (row[i] - mean);
        var /= (float)d;
        const float inv = 1.f / sqrtf(var + eps);
        for (size_t i = 0; i < d; ++i) row[i] = (row[i] - mean) * inv * w[i] + b[i];
    }
}

void oracle_gelu(float *x, size_t n) {
    for (size_t i = 0; i < n; ++i) x[i] = 0.5f * x[i] * (1.f + erff(x[i] * 0.70710678118654752440f));
}

int oracle_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
void oracle_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
