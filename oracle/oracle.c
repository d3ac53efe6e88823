/*
 * CPU oracle — TEST INFRASTRUCTURE ONLY (see oracle.h). Each function names
 * the reference file:line whose arithmetic it restates. Paths are relative
 * to the reference project (plainsight-systems/charlotte).
 *
 * Build: oracle/Makefile (-O3 -ffp-contract=off -fopenmp), so that only the
 * explicit fmaf() calls below fuse, exactly as the CUDA kernels fuse them.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* ---- scalar numerics ---------------------------------------------------- */

/* Exact binary16 -> binary32, subnormals kept (src/core/quant/q4_0.h:66). */
float or_fp16_to_fp32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    if (e == 0x1Fu) return u2f(sign | 0x7F800000u | (m << 13));
    if (e != 0) return u2f(sign | ((e + 112u) << 23) | (m << 13));
    if (m == 0) return u2f(sign);
    /* subnormal: m * 2^-24, exact */
    float v = (float)m * 0x1p-24f;
    return sign ? -v : v;
}

/* Saturate to +-65,504, then round to nearest even binary16
 * (formats/f16/f16_pack.wgsl:9-15; tests/support/f16_reference.h). */
uint16_t or_fp32_to_fp16_sat(float f) {
    uint32_t b = f2u(f);
    uint16_t sign = (uint16_t)((b >> 16) & 0x8000u);
    uint32_t mag = b & 0x7FFFFFFFu;
    if (mag > 0x7F800000u) return (uint16_t)(sign | 0x7E00u); /* NaN: never an input */
    if (u2f(mag) >= 65504.0f) return (uint16_t)(sign | 0x7BFFu);
    if (mag < 0x38800000u) { /* below 2^-14: result is an integer count of 2^-24 */
        float scaled = u2f(mag) * 0x1p24f; /* exact */
        return (uint16_t)(sign | (uint16_t)rintf(scaled));
    }
    uint32_t rounded = mag + 0x0FFFu + ((mag >> 13) & 1u);
    return (uint16_t)(sign | (uint16_t)((rounded >> 13) - (112u << 10)));
}

/* p * 2^k by multiplies with exact powers of two, two steps below 2^-126:
 * the definition of WGSL's ldexp used on both sides. */
float or_scale2(float p, int k) {
    while (k < -126) { p = p * 0x1p-64f; k += 64; }
    while (k > 127) { p = p * 0x1p64f; k -= 64; }
    return p * u2f((uint32_t)(k + 127) << 23);
}

/* e^x for x <= 0 (matmul.wgsl:169-182): Cody-Waite reduction by ln 2 in two
 * parts, Taylor series to r^6 in Horner form with fmas, then 2^k. */
float or_exp_nonpositive(float x) {
    float xc = fmaxf(x, -100.0f);
    float k = floorf(fmaf(xc, 1.4426950408889634f, 0.5f));
    float r = fmaf(k, -0.693145751953125f, xc);
    r = fmaf(k, -1.4286068203094172e-06f, r);
    float p = 1.0f / 720.0f;
    p = fmaf(p, r, 1.0f / 120.0f);
    p = fmaf(p, r, 1.0f / 24.0f);
    p = fmaf(p, r, 1.0f / 6.0f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    return or_scale2(p, (int)k);
}

/* SiLU, GELU (tanh form) and the sigmoid from e^x of a non-positive x
 * (matmul.wgsl:189-205). */
float or_activate(int activation, float g) {
    if (activation == OR_SILU) {
        float e = or_exp_nonpositive(-fabsf(g));
        float r = 1.0f / (1.0f + e);
        return g * (g >= 0.0f ? r : e * r);
    }
    if (activation == OR_SIGMOID) {
        float e = or_exp_nonpositive(-fabsf(g));
        float r = 1.0f / (1.0f + e);
        return g >= 0.0f ? r : e * r;
    }
    float z = 0.7978845608028654f * fmaf(0.044715f * g * g, g, g);
    float e = or_exp_nonpositive(-2.0f * fabsf(z));
    float sgn = z > 0.0f ? 1.0f : (z < 0.0f ? -1.0f : 0.0f);
    float t = sgn * ((1.0f - e) * (1.0f / (1.0f + e)));
    float half_g = 0.5f * g;
    return fmaf(half_g, t, half_g);
}

/* 2^x for x <= 0 — attention's exp2 (attention.wgsl:101-104, 262-273).
 * Method: x = k + r, k the nearest integer, r in [-1/2, 1/2] exact; 2^r =
 * e^(r ln 2) by its Taylor series to degree 7 (truncation under 6e-9
 * relative for |r ln 2| <= 0.347), Horner with fmas; then 2^k exactly. */
float or_exp2(float x) {
    float xc = fmaxf(x, -160.0f);
    float k = floorf(xc + 0.5f);
    float r = xc - k;
    float t = r * 0.693147182f;
    float p = 1.0f / 5040.0f;
    p = fmaf(p, t, 1.0f / 720.0f);
    p = fmaf(p, t, 1.0f / 120.0f);
    p = fmaf(p, t, 1.0f / 24.0f);
    p = fmaf(p, t, 1.0f / 6.0f);
    p = fmaf(p, t, 0.5f);
    p = fmaf(p, t, 1.0f);
    p = fmaf(p, t, 1.0f);
    return or_scale2(p, (int)k);
}

/* sin and cos of an angle in [-pi, pi] (rope.wgsl:94-99). Method (Cody and
 * Waite): q = the nearest integer to angle * 2/pi, r = angle - q * pi/2 with
 * pi/2 in two parts, |r| <= pi/4 + tiny; sin r and cos r by their Taylor
 * series to r^9 and r^10 (truncation under 2e-9), Horner in r^2 with fmas;
 * then the quadrant q mod 4 picks and signs them. */
void or_sincos(float angle, float* s_out, float* c_out) {
    float q = rintf(angle * 0.636619772f);
    float r = fmaf(q, -1.57079625f, angle);
    r = fmaf(q, -7.54978942e-08f, r);
    float r2 = r * r;
    float ps = -1.0f / 39916800.0f;
    ps = fmaf(ps, r2, 1.0f / 362880.0f);
    ps = fmaf(ps, r2, -1.0f / 5040.0f);
    ps = fmaf(ps, r2, 1.0f / 120.0f);
    ps = fmaf(ps, r2, -1.0f / 6.0f);
    float s = fmaf(ps * r2, r, r);
    float pc = 1.0f / 3628800.0f;
    pc = fmaf(pc, r2, -1.0f / 40320.0f);
    pc = fmaf(pc, r2, 1.0f / 720.0f);
    pc = fmaf(pc, r2, -1.0f / 24.0f);
    pc = fmaf(pc, r2, 0.5f);
    float c = fmaf(-pc, r2, 1.0f);
    int quadrant = ((int)q) & 3;
    float so, co;
    switch (quadrant) {
        case 0: so = s; co = c; break;
        case 1: so = c; co = -s; break;
        case 2: so = -s; co = -c; break;
        default: so = -c; co = s; break;
    }
    *s_out = so;
    *c_out = co;
}

float or_dot4(const float* a, const float* b) {
    return fmaf(a[3], b[3], fmaf(a[2], b[2], fmaf(a[1], b[1], a[0] * b[0])));
}

/* ---- formats ------------------------------------------------------------- */

uint32_t or_block_bytes(int type) {
    switch (type) {
        case OR_F32: return 4;
        case OR_F16: return 2;
        case OR_Q4_0: return 18;
        case OR_Q4_1: return 20;
        case OR_BF16: return 2;
        case OR_Q8_0: return 34;
        case OR_Q6_K: return 210;
        default: return 0;
    }
}

uint32_t or_block_weights(int type) {
    switch (type) {
        case OR_F32: case OR_F16: case OR_BF16: return 1;
        case OR_Q4_0: case OR_Q4_1: case OR_Q8_0: return 32;
        case OR_Q6_K: return 256;
        default: return 0;
    }
}

static inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* ggml's dequantize_row_* order (tests/support/q4_0_reference.h:25,
 * q8_0_reference.h:15, q6_k_reference.h:17). */
int or_dequant_stored(int type, const uint8_t* data, size_t blocks, float* out) {
    size_t b;
    switch (type) {
        case OR_Q4_0:
            for (b = 0; b < blocks; ++b) {
                const uint8_t* blk = data + b * 18;
                float d = or_fp16_to_fp32(rd16(blk));
                for (int j = 0; j < 16; ++j) {
                    out[b * 32 + j] = (float)((int)(blk[2 + j] & 0x0F) - 8) * d;
                    out[b * 32 + j + 16] = (float)((int)(blk[2 + j] >> 4) - 8) * d;
                }
            }
            return 0;
        case OR_Q8_0:
            for (b = 0; b < blocks; ++b) {
                const uint8_t* blk = data + b * 34;
                float d = or_fp16_to_fp32(rd16(blk));
                for (int j = 0; j < 32; ++j) out[b * 32 + j] = (float)(int8_t)blk[2 + j] * d;
            }
            return 0;
        case OR_Q4_1:   /* q4_1_reference.h:44-50, the fused evaluation: fma(q, d, m) */
            for (b = 0; b < blocks; ++b) {
                const uint8_t* blk = data + b * 20;
                float d = or_fp16_to_fp32(rd16(blk)), m = or_fp16_to_fp32(rd16(blk + 2));
                for (int j = 0; j < 16; ++j) {
                    out[b * 32 + j] = fmaf((float)(blk[4 + j] & 0x0F), d, m);
                    out[b * 32 + j + 16] = fmaf((float)(blk[4 + j] >> 4), d, m);
                }
            }
            return 0;
        case OR_BF16:   /* the top half of an f32 (bf16.wgsl) */
            for (b = 0; b < blocks; ++b) {
                uint32_t bits = (uint32_t)rd16(data + 2 * b) << 16;
                memcpy(out + b, &bits, 4);
            }
            return 0;
        case OR_Q6_K:
            for (b = 0; b < blocks; ++b) {
                const uint8_t* blk = data + b * 210;
                float d = or_fp16_to_fp32(rd16(blk + 208));
                for (int k = 0; k < 8; ++k) {
                    int h = k / 4, r = k % 4;
                    for (int l = 0; l < 32; ++l) {
                        int lo = (blk[64 * h + 32 * (r % 2) + l] >> (4 * (r / 2))) & 0xF;
                        int hi = (blk[128 + 32 * h + l] >> (2 * r)) & 3;
                        int q = (lo | (hi << 4)) - 32;
                        float sc = (float)(int8_t)blk[192 + 2 * k + l / 16];
                        out[b * 256 + 32 * k + l] = d * sc * (float)q;
                    }
                }
            }
            return 0;
        case OR_F32:
            memcpy(out, data, blocks * 4);
            return 0;
        case OR_F16:
            for (b = 0; b < blocks; ++b) out[b] = or_fp16_to_fp32(rd16(data + 2 * b));
            return 0;
        default:
            return -1;
    }
}

size_t or_piece_bytes(int type, size_t blocks) {
    size_t stored = blocks * or_block_bytes(type);
    return (stored + 15) & ~(size_t)15;
}

/* device_layout.h:121-136: streams in device order; Q6_K repacked per
 * q6_k.h:9-21 (low nibbles of group k at 16k, byte j = weight j's nibble
 * then weight j+16's; high pairs at 8k, byte m = weights m, m+8, m+16,
 * m+24 from bit 0 up; scales and d as stored). */
int or_to_piece(int type, const uint8_t* stored, size_t blocks, uint8_t* piece) {
    size_t total = or_piece_bytes(type, blocks);
    memset(piece, 0, total);
    size_t b;
    switch (type) {
        case OR_Q4_0:
            for (b = 0; b < blocks; ++b) {
                memcpy(piece + 16 * b, stored + 18 * b + 2, 16);
                memcpy(piece + 16 * blocks + 2 * b, stored + 18 * b, 2);
            }
            return 0;
        case OR_Q8_0:
            for (b = 0; b < blocks; ++b) {
                memcpy(piece + 32 * b, stored + 34 * b + 2, 32);
                memcpy(piece + 32 * blocks + 2 * b, stored + 34 * b, 2);
            }
            return 0;
        case OR_Q6_K:
            for (b = 0; b < blocks; ++b) {
                const uint8_t* blk = stored + 210 * b;
                uint8_t* lo = piece + 128 * b;
                uint8_t* hi = piece + 128 * blocks + 64 * b;
                for (int k = 0; k < 8; ++k) {
                    int h = k / 4, r = k % 4;
                    for (int l = 0; l < 32; ++l) {
                        int nib = (blk[64 * h + 32 * (r % 2) + l] >> (4 * (r / 2))) & 0xF;
                        int pair = (blk[128 + 32 * h + l] >> (2 * r)) & 3;
                        lo[16 * k + l % 16] |= (uint8_t)(nib << (4 * (l / 16)));
                        hi[8 * k + l % 8] |= (uint8_t)(pair << (2 * (l / 8)));
                    }
                }
                memcpy(piece + 192 * blocks + 16 * b, blk + 192, 16);
                memcpy(piece + 208 * blocks + 2 * b, blk + 208, 2);
            }
            return 0;
        case OR_Q4_1:   /* codes, then each block's (d, m) word (device_layout.h:122) */
            for (b = 0; b < blocks; ++b) {
                memcpy(piece + 16 * b, stored + 20 * b + 4, 16);
                memcpy(piece + 16 * blocks + 4 * b, stored + 20 * b, 4);
            }
            return 0;
        case OR_F32: case OR_F16: case OR_BF16:
            memcpy(piece, stored, blocks * or_block_bytes(type));
            return 0;
        default:
            return -1;
    }
}

/* Each format's unpack (q4_0.wgsl:6-18, q8_0.wgsl:6-17, q6_k.wgsl:13-42,
 * f32.wgsl, f16.wgsl). */
int or_unpack(int type, const uint8_t* piece, uint32_t n, uint32_t group, float* out) {
    switch (type) {
        case OR_Q4_0: {
            float d = or_fp16_to_fp32(rd16(piece + (size_t)16 * n + 2 * (size_t)group));
            const uint8_t* qs = piece + (size_t)16 * group;
            for (int j = 0; j < 16; ++j) {
                out[j] = ((float)(qs[j] & 0xF) - 8.0f) * d;
                out[j + 16] = ((float)(qs[j] >> 4) - 8.0f) * d;
            }
            return 0;
        }
        case OR_Q8_0: {
            float d = or_fp16_to_fp32(rd16(piece + (size_t)32 * n + 2 * (size_t)group));
            const uint8_t* qs = piece + (size_t)32 * group;
            for (int j = 0; j < 32; ++j) out[j] = (float)(int8_t)qs[j] * d;
            return 0;
        }
        case OR_Q6_K: {
            uint32_t b = group / 8, k = group % 8;
            float d = or_fp16_to_fp32(rd16(piece + (size_t)208 * n + 2 * (size_t)b));
            const uint8_t* sc = piece + (size_t)192 * n + 16 * (size_t)b + 2 * k;
            float first = d * (float)(int8_t)sc[0];
            float second = d * (float)(int8_t)sc[1];
            const uint8_t* lo = piece + (size_t)128 * b + 16 * k;
            const uint8_t* hi = piece + (size_t)128 * n + (size_t)64 * b + 8 * k;
            for (int l = 0; l < 32; ++l) {
                int q = ((lo[l % 16] >> (4 * (l / 16))) & 0xF) | (((hi[l % 8] >> (2 * (l / 8))) & 3) << 4);
                out[l] = (l < 16 ? first : second) * (float)(q - 32);
            }
            return 0;
        }
        case OR_F32:
            memcpy(out, piece + (size_t)128 * group, 128);
            return 0;
        case OR_F16:
            for (int j = 0; j < 32; ++j) out[j] = or_fp16_to_fp32(rd16(piece + (size_t)64 * group + 2 * j));
            return 0;
        case OR_Q4_1: {   /* q4_1.wgsl:6-20, fused: fma(q, d, m) */
            const uint8_t* dm = piece + (size_t)16 * n + 4 * (size_t)group;
            float d = or_fp16_to_fp32(rd16(dm)), m = or_fp16_to_fp32(rd16(dm + 2));
            const uint8_t* qs = piece + (size_t)16 * group;
            for (int j = 0; j < 16; ++j) {
                out[j] = fmaf((float)(qs[j] & 0xF), d, m);
                out[j + 16] = fmaf((float)(qs[j] >> 4), d, m);
            }
            return 0;
        }
        case OR_BF16:   /* bf16.wgsl:9-20 */
            for (int j = 0; j < 32; ++j) {
                uint32_t bits = (uint32_t)rd16(piece + (size_t)64 * group + 2 * j) << 16;
                memcpy(out + j, &bits, 4);
            }
            return 0;
        default:
            return -1;
    }
}

/* ---- matrix products ----------------------------------------------------- */

#define OR_RANGES 32
#define OR_ROWBLOCK 8

/* y = W x in the order decode_ranges (matmul.wgsl:212-234), slot_total
 * (:237-243) and the tiled form (tile_range :410, prefill_tile :480) share:
 * the row's G = K/32 groups cut into 32 ranges at floor(r*G/32); each range
 * an fma chain from zero over its weights in order; the ranges added to a
 * total from zero, in order (matmul.h:34-50). Rows are worked 8 at a time,
 * each row's chain its own, so the compiler may vectorize across rows
 * without changing any row's order. */
int or_matmul(int type, const uint8_t* piece, uint32_t blocks_in_piece, uint32_t row0, uint32_t rows,
              uint32_t K, const float* x, uint32_t tokens, float* y, uint32_t y_stride, int threads) {
    if (K % 32 != 0 || or_block_bytes(type) == 0) return -1;
    const uint32_t G = K / 32;
    const int64_t blocks_of_rows = (rows + OR_ROWBLOCK - 1) / OR_ROWBLOCK;
    int64_t rb;
#ifdef _OPENMP
    if (threads < 1) threads = 1;
#pragma omp parallel for num_threads(threads) schedule(dynamic, 4)
#endif
    for (rb = 0; rb < blocks_of_rows; ++rb) {
        float w[OR_ROWBLOCK][32];
        const uint32_t o0 = (uint32_t)rb * OR_ROWBLOCK;
        const uint32_t nrow = rows - o0 < OR_ROWBLOCK ? rows - o0 : OR_ROWBLOCK;
        for (uint32_t t = 0; t < tokens; ++t) {
            const float* xt = x + (size_t)t * K;
            float total[OR_ROWBLOCK] = {0};
            for (uint32_t r = 0; r < OR_RANGES; ++r) {
                const uint32_t lo = r * G / OR_RANGES, hi = (r + 1) * G / OR_RANGES;
                float s[OR_ROWBLOCK] = {0};
                for (uint32_t g = lo; g < hi; ++g) {
                    for (uint32_t i = 0; i < OR_ROWBLOCK; ++i) {
                        if (i < nrow) or_unpack(type, piece, blocks_in_piece, (row0 + o0 + i) * G + g, w[i]);
                        else memset(w[i], 0, sizeof w[i]);
                    }
                    const float* xg = xt + (size_t)g * 32;
                    for (int k = 0; k < 32; ++k) {
                        const float xk = xg[k];
                        for (int i = 0; i < OR_ROWBLOCK; ++i) s[i] = fmaf(w[i][k], xk, s[i]);
                    }
                }
                for (int i = 0; i < OR_ROWBLOCK; ++i) total[i] = total[i] + s[i];
            }
            for (uint32_t i = 0; i < nrow; ++i) y[(size_t)t * y_stride + o0 + i] = total[i];
        }
    }
    return 0;
}

/* ---- norm ---------------------------------------------------------------- */

#define OR_NORM_WG 256

/* reduce (norm.wgsl:67-78): 256 partial sums halved level by level. */
static float norm_reduce(float* partial) {
    for (int stride = OR_NORM_WG / 2; stride > 0; stride /= 2)
        for (int i = 0; i < stride; ++i) partial[i] = partial[i] + partial[i + stride];
    return partial[0];
}

/* The sum of squares as invocation i of 256 sums vec4s i, i+256, ... with
 * `squares + dot`, then the tree. */
static float norm_squares(const float* x, uint32_t width) {
    float partial[OR_NORM_WG];
    uint32_t vec4s = width / 4;
    for (uint32_t i = 0; i < OR_NORM_WG; ++i) {
        float squares = 0.0f;
        for (uint32_t v = i; v < vec4s; v += OR_NORM_WG) squares = squares + or_dot4(x + 4 * v, x + 4 * v);
        partial[i] = squares;
    }
    return norm_reduce(partial);
}

/* norm.wgsl:80-198 for one row (Rows::EveryToken or the final norm's last
 * row): the add (post-norm of y first, Gemma 3), then normed = (x*r)*g. */
void or_norm_row(float* hidden, const float* output, const float* gain, const float* post_gain, uint32_t width,
                 float epsilon, int add, float* normed) {
    const float n = (float)width;
    if (add) {
        float y[4096];
        memcpy(y, output, width * sizeof(float));
        if (post_gain) {
            float r = 1.0f / sqrtf(norm_squares(y, width) / n + epsilon);
            for (uint32_t j = 0; j < width; ++j) y[j] = ((y[j] * r) * post_gain[j]) * 1.0f;
        }
        for (uint32_t j = 0; j < width; ++j) hidden[j] = hidden[j] + y[j];
    }
    float r = 1.0f / sqrtf(norm_squares(hidden, width) / n + epsilon);
    for (uint32_t j = 0; j < width; ++j) normed[j] = (hidden[j] * r) * gain[j];
}

/* ---- rope ------------------------------------------------------------------ */

/* constants_of (rope.cpp:76-87): theta_k / 2pi in f64, rounded once. */
void or_rope_turns(double base, uint32_t head_dim, float* turns) {
    for (uint32_t k = 0; k < head_dim / 2; ++k) {
        double theta = pow(base, -2.0 * k / head_dim);
        turns[k] = (float)(theta / (2 * 3.14159265358979323846));
    }
}

/* reduce_head (rope.wgsl:62-73) over `lanes` partials. */
static float head_reduce(float* partial, uint32_t lanes) {
    for (uint32_t stride = lanes / 2; stride > 0; stride /= 2)
        for (uint32_t i = 0; i < stride; ++i) partial[i] = partial[i] + partial[i + stride];
    return partial[0];
}

static void norm_head(float* x, uint32_t d, const float* gain, float epsilon) {
    const uint32_t lanes = d / 8;
    float partial[64];
    for (uint32_t i = 0; i < lanes; ++i)
        partial[i] = or_dot4(x + 4 * i, x + 4 * i) + or_dot4(x + 4 * (i + lanes), x + 4 * (i + lanes));
    float total = head_reduce(partial, lanes);
    float r = 1.0f / sqrtf(total / (float)d + epsilon);
    for (uint32_t j = 0; j < d; ++j) x[j] = (x[j] * r) * gain[j];
}

/* rotate (rope.wgsl:140-156). */
static void rotate_head(float* x, uint32_t d, int halves, const float* cosines, const float* sines) {
    if (halves) {
        for (uint32_t k = 0; k < d / 2; ++k) {
            float a = x[k], b = x[k + d / 2];
            x[k] = fmaf(a, cosines[k], -(b * sines[k]));
            x[k + d / 2] = fmaf(a, sines[k], b * cosines[k]);
        }
    } else {
        for (uint32_t k = 0; k < d / 2; ++k) {
            float a = x[2 * k], b = x[2 * k + 1];
            x[2 * k] = fmaf(a, cosines[k], (-b) * sines[k]);
            x[2 * k + 1] = fmaf(b, cosines[k], a * sines[k]);
        }
    }
}

/* rope_cache.wgsl:11-89 with rope.wgsl's angles (:86-100): one token. */
void or_rope_token(const or_rope_shape* s, uint32_t p, float* q, const float* k, const float* v,
                   uint16_t* key_cache, uint16_t* value_cache) {
    const uint32_t d = s->head_dim;
    float cosines[256], sines[256];
    for (uint32_t j = 0; j < d / 2; ++j) {
        float t = (float)p * s->turns[j];
        if (s->factors) t = t / s->factors[j];
        float angle = 6.283185307179586f * (t - rintf(t));
        or_sincos(angle, &sines[j], &cosines[j]);
    }
    float kh[512];
    for (uint32_t h = 0; h < s->query_heads; ++h) {
        float* x = q + (size_t)h * d;
        if (s->qk_norm) norm_head(x, d, s->query_gain, s->epsilon);
        rotate_head(x, d, s->halves, cosines, sines);
    }
    const size_t slot = (size_t)(p % s->slots) * s->kv_heads * d;
    for (uint32_t h = 0; h < s->kv_heads; ++h) {
        memcpy(kh, k + (size_t)h * d, d * sizeof(float));
        if (s->qk_norm) norm_head(kh, d, s->key_gain, s->epsilon);
        rotate_head(kh, d, s->halves, cosines, sines);
        for (uint32_t j = 0; j < d; ++j) {
            key_cache[slot + (size_t)h * d + j] = or_fp32_to_fp16_sat(kh[j]);
            value_cache[slot + (size_t)h * d + j] = or_fp32_to_fp16_sat(v[(size_t)h * d + j]);
        }
    }
}

/* ---- an encoder's kernels --------------------------------------------------- */

/* norm.wgsl:80-198 with the `scaled`, `normalize`, post_scale and unit-gain
 * variants (norm.h:69-99), one row. */
void or_norm_row_ex(float* hidden, const float* output, const float* gain, const float* post_gain, float post_scale,
                    const float* scale, uint32_t width, float epsilon, int add, int normalize, float* normed) {
    const float n = (float)width;
    if (add) {
        float y[4096];
        memcpy(y, output, width * sizeof(float));
        if (post_gain) {
            float r = 1.0f / sqrtf(norm_squares(y, width) / n + epsilon);
            for (uint32_t j = 0; j < width; ++j) y[j] = ((y[j] * r) * post_gain[j]) * post_scale;
        }
        const float s = scale ? scale[0] : 1.0f;
        for (uint32_t j = 0; j < width; ++j) {
            float x = hidden[j] + y[j];
            if (scale) x = x * s;
            hidden[j] = x;
        }
    }
    if (!normalize) return;
    float r = 1.0f / sqrtf(norm_squares(hidden, width) / n + epsilon);
    for (uint32_t j = 0; j < width; ++j) normed[j] = gain ? (hidden[j] * r) * gain[j] : hidden[j] * r;
}

/* rope_encode.wgsl:8-76: the decoder form's angles, QK-norm and turn, every
 * head in place; value heads x·r with value_norm (the head's reduce_head,
 * no gain), not turned. */
void or_rope_encode_token(const or_rope_shape* s, uint32_t p, int value_norm, float* q, float* k, float* v) {
    const uint32_t d = s->head_dim;
    float cosines[256], sines[256];
    for (uint32_t j = 0; j < d / 2; ++j) {
        float t = (float)p * s->turns[j];
        if (s->factors) t = t / s->factors[j];
        float angle = 6.283185307179586f * (t - rintf(t));
        or_sincos(angle, &sines[j], &cosines[j]);
    }
    for (uint32_t h = 0; h < s->query_heads; ++h) {
        float* x = q + (size_t)h * d;
        if (s->qk_norm) norm_head(x, d, s->query_gain, s->epsilon);
        rotate_head(x, d, s->halves, cosines, sines);
    }
    for (uint32_t h = 0; h < s->kv_heads; ++h) {
        float* x = k + (size_t)h * d;
        if (s->qk_norm) norm_head(x, d, s->key_gain, s->epsilon);
        rotate_head(x, d, s->halves, cosines, sines);
    }
    if (value_norm) {
        const uint32_t lanes = d / 8;
        for (uint32_t h = 0; h < s->kv_heads; ++h) {
            float* x = v + (size_t)h * d;
            float partial[64];
            for (uint32_t i = 0; i < lanes; ++i)
                partial[i] = or_dot4(x + 4 * i, x + 4 * i) + or_dot4(x + 4 * (i + lanes), x + 4 * (i + lanes));
            float r = 1.0f / sqrtf(head_reduce(partial, lanes) / (float)d + s->epsilon);
            for (uint32_t j = 0; j < d; ++j) x[j] = x[j] * r;
        }
    }
}

/* block_attention.wgsl: scores_of (:95-190) — s_ij = (the chain of dot4s
 * along d in order) × scale·log2e — and weigh (:205-326) — m the largest live
 * score of the row, p = exp2(s − m) for live keys, O = fma(p, v, O) and
 * l = l + p in key order, out = O / l. A key not live adds an exact zero
 * (fma(0, v, O) = O; O is never −0), so it is skipped here. */
void or_block_attention(const float* q, const float* k, const float* v, uint32_t n, uint32_t d, uint32_t query_heads,
                        uint32_t kv_heads, uint32_t half_window, float scale_log2e, float* out) {
    const uint32_t G = query_heads / kv_heads;
    float* s = (float*)malloc((size_t)n * sizeof(float));
    float o[512];
    for (uint32_t i = 0; i < n; ++i) {
        const uint32_t lo = i > half_window ? i - half_window : 0;
        const uint32_t hi = i + half_window < n - 1 ? i + half_window : n - 1;
        for (uint32_t h = 0; h < query_heads; ++h) {
            const uint32_t kv = h / G;
            const float* qv = q + ((size_t)i * query_heads + h) * d;
            float m = 0.0f;
            int seen = 0;
            for (uint32_t j = lo; j <= hi; ++j) {
                const float* kj = k + ((size_t)j * kv_heads + kv) * d;
                float acc = 0.0f;
                for (uint32_t c = 0; c < d; c += 4) acc = acc + or_dot4(qv + c, kj + c);
                s[j] = acc * scale_log2e;
                m = seen ? fmaxf(m, s[j]) : s[j];
                seen = 1;
            }
            float l = 0.0f;
            for (uint32_t c = 0; c < d; ++c) o[c] = 0.0f;
            for (uint32_t j = lo; j <= hi; ++j) {
                const float p = or_exp2(s[j] - m);
                const float* vj = v + ((size_t)j * kv_heads + kv) * d;
                for (uint32_t c = 0; c < d; ++c) o[c] = fmaf(p, vj[c], o[c]);
                l = l + p;
            }
            float* dst = out + ((size_t)i * query_heads + h) * d;
            for (uint32_t c = 0; c < d; ++c) dst[c] = o[c] / l;
        }
    }
    free(s);
}

/* pool.wgsl mean (:49-61) and unit (:63-100). */
void or_pool_mean(const float* rows, uint32_t n, uint32_t width, float* mean) {
    const float inverse = 1.0f / (float)n;
    for (uint32_t c = 0; c < width; ++c) {
        float sum = 0.0f;
        for (uint32_t r = 0; r < n; ++r) sum = sum + rows[(size_t)r * width + c];
        mean[c] = sum * inverse;
    }
}

void or_pool_unit(const float* row, uint32_t width, float* unit) {
    float partial[OR_NORM_WG];
    const uint32_t vec4s = width / 4;
    for (uint32_t i = 0; i < OR_NORM_WG; ++i) {
        float squares = 0.0f;
        for (uint32_t c = i; c < vec4s; c += OR_NORM_WG) squares = squares + or_dot4(row + 4 * c, row + 4 * c);
        partial[i] = squares;
    }
    const float total = norm_reduce(partial);
    const float r = total > 0.0f ? 1.0f / sqrtf(total) : 0.0f;
    for (uint32_t c = 0; c < width; ++c) unit[c] = row[c] * r;
}

/* ---- attention ------------------------------------------------------------- */

#define OR_CHUNK_KEYS 64

/* attention.wgsl:138-360 (main) and :363-392 (combine) for one query row:
 * per head, chunks of 64 keys fixed by position, each an online softmax over
 * tiles of B = 2048/d keys aligned to B, folded into the running state in
 * chunk order with fold_factors/fold_sum/fold (:101-127). Keys not live for
 * the query (causal, window) contribute exactly nothing in the reference
 * (a multiply by a zero weight added to a non-negative-zero sum), so they are
 * skipped here; a chunk or tile with no live key leaves the state's bits as
 * they were. */
void or_attention_row(const float* q_in, uint32_t p, const uint16_t* key_cache, const uint16_t* value_cache,
                      uint32_t slots, uint32_t window, float scale_log2e, uint32_t d, uint32_t query_heads,
                      uint32_t kv_heads, float* out) {
    const uint32_t B = 2048 / d;
    const uint32_t G = query_heads / kv_heads;
    const uint32_t earliest = p + 1 > window ? p + 1 - window : 0;
    float q[512], o_chunk[512], o_run[512], s_tile[64], p_tile[64];
    for (uint32_t h = 0; h < query_heads; ++h) {
        const uint32_t kv = h / G;
        for (uint32_t j = 0; j < d; ++j) q[j] = q_in[(size_t)h * d + j] * scale_log2e;
        int run_live = 0;
        float run_m = 0.0f, run_l = 0.0f;
        for (uint32_t j = 0; j < d; ++j) o_run[j] = 0.0f;
        for (uint32_t c = earliest / OR_CHUNK_KEYS; c <= p / OR_CHUNK_KEYS; ++c) {
            int chunk_live = 0;
            float chunk_m = 0.0f, chunk_l = 0.0f;
            for (uint32_t j = 0; j < d; ++j) o_chunk[j] = 0.0f;
            uint32_t k_begin = c * OR_CHUNK_KEYS;
            uint32_t aligned = earliest / B * B;
            if (aligned > k_begin) k_begin = aligned;
            uint32_t k_end = (c + 1) * OR_CHUNK_KEYS;
            if (p + 1 < k_end) k_end = p + 1;
            for (uint32_t j0 = k_begin; j0 < k_end; j0 += B) {
                float top_tile = 0.0f;
                int seen = 0;
                for (uint32_t b = 0; b < B; ++b) {
                    uint32_t j = j0 + b;
                    int live = j < k_end && j <= p && j >= earliest;
                    float s = 0.0f;
                    if (live) {
                        const uint16_t* kr = key_cache + ((size_t)(j % slots) * kv_heads + kv) * d;
                        for (uint32_t w = 0; w < d / 4; ++w) {
                            float kk[4] = {or_fp16_to_fp32(kr[4 * w]), or_fp16_to_fp32(kr[4 * w + 1]),
                                           or_fp16_to_fp32(kr[4 * w + 2]), or_fp16_to_fp32(kr[4 * w + 3])};
                            s = s + or_dot4(q + 4 * w, kk);
                        }
                        top_tile = seen ? fmaxf(top_tile, s) : s;
                        seen = 1;
                    }
                    s_tile[b] = live ? s : 0.0f;
                    p_tile[b] = live ? 1.0f : 0.0f; /* liveness, for phase 3 */
                }
                float a = 1.0f;
                if (seen) {
                    float old = chunk_live ? chunk_m : top_tile;
                    chunk_live = 1;
                    float top = fmaxf(old, top_tile);
                    a = old == top ? 1.0f : or_exp2(old - top);
                    float sum = 0.0f;
                    for (uint32_t b = 0; b < B; ++b) {
                        float e = 0.0f;
                        if (p_tile[b] != 0.0f) e = or_exp2(s_tile[b] - top);
                        p_tile[b] = e;
                        sum = sum + e;
                    }
                    chunk_l = fmaf(chunk_l, a, sum);
                    chunk_m = top;
                } else {
                    for (uint32_t b = 0; b < B; ++b) p_tile[b] = 0.0f;
                }
                for (uint32_t jj = 0; jj < d; ++jj) o_chunk[jj] = o_chunk[jj] * a;
                for (uint32_t b = 0; b < B; ++b) {
                    if (p_tile[b] == 0.0f) continue;
                    const uint16_t* vr = value_cache + ((size_t)((j0 + b) % slots) * kv_heads + kv) * d;
                    for (uint32_t jj = 0; jj < d; ++jj) o_chunk[jj] = fmaf(p_tile[b], or_fp16_to_fp32(vr[jj]), o_chunk[jj]);
                }
            }
            /* fold_factors (:101-116), fold_sum, fold (:118-124) */
            if (!chunk_live) continue;
            float fa, fb, fm;
            if (!run_live) { fa = 0.0f; fb = 1.0f; fm = chunk_m; }
            else if (run_m == chunk_m) { fa = 1.0f; fb = 1.0f; fm = run_m; }
            else if (run_m > chunk_m) { fa = 1.0f; fb = or_exp2(chunk_m - run_m); fm = run_m; }
            else { fa = or_exp2(run_m - chunk_m); fb = 1.0f; fm = chunk_m; }
            run_l = fmaf(run_l, fa, chunk_l * fb);
            for (uint32_t jj = 0; jj < d; ++jj) o_run[jj] = fmaf(o_run[jj], fa, o_chunk[jj] * fb);
            run_m = fm;
            run_live = 1;
        }
        for (uint32_t jj = 0; jj < d; ++jj) out[(size_t)h * d + jj] = run_live ? o_run[jj] / run_l : 0.0f;
    }
}

/* ---- selection and draw ---------------------------------------------------- */

uint32_t or_key_of(uint32_t b) {
    if (b == 0x80000000u) b = 0u;
    if ((b & 0x7F800000u) == 0x7F800000u && (b & 0x007FFFFFu) != 0u) return 0xFFFFFFFFu;
    if (b & 0x80000000u) return ~b;
    return b | 0x80000000u;
}

uint32_t or_bits_of(uint32_t key) {
    if (key == 0xFFFFFFFFu) return 0x7FC00000u;
    if (key & 0x80000000u) return key & 0x7FFFFFFFu;
    return ~key;
}

typedef struct { uint32_t key, id; } or_entry;

static int entry_before(const void* pa, const void* pb) {
    const or_entry* a = (const or_entry*)pa;
    const or_entry* b = (const or_entry*)pb;
    if (a->key != b->key) return a->key > b->key ? -1 : 1;
    if (a->id != b->id) return a->id < b->id ? -1 : 1;
    return 0;
}

/* The top 64 under topk.wgsl's total order (before :55: larger key, then
 * lower token), as its three passes leave them in `candidates`. */
void or_topk64(const float* logits, uint32_t count, uint32_t* pairs) {
    or_entry* e = (or_entry*)malloc((count ? count : 1) * sizeof(or_entry));
    for (uint32_t i = 0; i < count; ++i) {
        uint32_t bits;
        memcpy(&bits, logits + i, 4);
        e[i].key = or_key_of(bits);
        e[i].id = i;
    }
    qsort(e, count, sizeof(or_entry), entry_before);
    for (uint32_t i = 0; i < 64; ++i) {
        if (i < count) { pairs[2 * i] = or_bits_of(e[i].key); pairs[2 * i + 1] = e[i].id; }
        else { pairs[2 * i] = 0xFFFFFFFFu; pairs[2 * i + 1] = 0xFFFFFFFFu; }
    }
    free(e);
}

/* Philox4x32-10 (Salmon et al., SC '11), Random123's multipliers and Weyl
 * constants, as draw.wgsl:41-52 runs it. */
void or_philox4x32_10(const uint32_t counter[4], const uint32_t key_in[2], uint32_t out[4]) {
    uint32_t c0 = counter[0], c1 = counter[1], c2 = counter[2], c3 = counter[3];
    uint32_t k0 = key_in[0], k1 = key_in[1];
    for (int r = 0; r < 10; ++r) {
        uint64_t p0 = (uint64_t)0xD2511F53u * c0;
        uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
        uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
        uint32_t n1 = (uint32_t)p1;
        uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
        uint32_t n3 = (uint32_t)p0;
        c0 = n0; c1 = n1; c2 = n2; c3 = n3;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

static int finite_bits(uint32_t b) { return (b & 0x7F800000u) != 0x7F800000u; }

/* draw.wgsl:71-163: top-k/top-p/min-p/temperature over the 64 candidates;
 * temperature 0 keeps candidate 0 (greedy). exp is or_exp_nonpositive: every
 * argument is <= 0. */
void or_draw(const uint32_t* cand, const or_draw_settings* st, uint32_t* record) {
    uint32_t k = st->top_k < 64 ? st->top_k : 64;
    if (k == 0) k = 1;
    int top_p = st->top_p < 1.0f;
    float weight[64], tempered[64], running[64];
    uint32_t above[64];
    uint32_t first_bits = cand[0];
    int failed = !finite_bits(first_bits);
    for (uint32_t t = 0; t < k; ++t) {
        weight[t] = 0.0f;
        tempered[t] = 0.0f;
        above[t] = 0;
        uint32_t mine_bits = cand[2 * t];
        if (!failed && mine_bits != 0xFF800000u) {
            float first, mine;
            memcpy(&first, &first_bits, 4);
            memcpy(&mine, &mine_bits, 4);
            if (top_p) weight[t] = or_exp_nonpositive(mine - first);
            if (st->temperature > 0.0f) tempered[t] = or_exp_nonpositive((mine - first) / st->temperature);
            above[t] = (st->min_p == 0.0f || mine >= first + st->log_min_p) ? 1u : 0u;
        }
    }
    uint32_t counter[4] = {st->position + st->tokens, 0, 0, 0};
    uint32_t key[2] = {st->seed0, st->seed1};
    uint32_t ph[4];
    or_philox4x32_10(counter, key, ph);
    float u = (float)(ph[0] >> 9) * (1.0f / 8388608.0f) + (1.0f / 16777216.0f);
    if (top_p) {
        float sum = 0.0f;
        for (uint32_t i = 0; i < k; ++i) sum = sum + weight[i];
        if (!failed)
            for (uint32_t i = 0; i < k; ++i) weight[i] = weight[i] / sum;
    }
    uint32_t kept = k;
    float cumulative = 0.0f, tempered_sum = 0.0f;
    for (uint32_t i = 0; i < k; ++i) {
        tempered_sum = tempered_sum + tempered[i];
        running[i] = tempered_sum;
        if (top_p) {
            cumulative = cumulative + weight[i];
            if (cumulative >= st->top_p) { kept = i + 1; break; }
        }
    }
    uint32_t survivors = 1;
    while (survivors < kept && above[survivors] == 1u) survivors++;
    uint32_t chosen = 0;
    if (st->temperature > 0.0f) {
        float goal = u * running[survivors - 1];
        chosen = survivors - 1;
        for (uint32_t i = 0; i < survivors; ++i)
            if (running[i] > goal) { chosen = i; break; }
    }
    record[0] = failed ? 0u : cand[2 * chosen + 1];
    record[1] = failed ? 1u : 0u;
    memcpy(&record[2], &u, 4);
    record[3] = 0u;
}

/* ---- whole decoder pass ---------------------------------------------------- */

struct or_state {
    const or_model* m;
    uint16_t** kcache;
    uint16_t** vcache;
    float *hidden, *normed, *q, *k, *v, *att, *out, *gate, *up, *act, *logits;
    int pending_add;
    const float* pending_post;
};

or_state* or_state_create(const or_model* m) {
    or_state* s = (or_state*)calloc(1, sizeof(or_state));
    s->m = m;
    s->kcache = (uint16_t**)calloc(m->layers, sizeof(uint16_t*));
    s->vcache = (uint16_t**)calloc(m->layers, sizeof(uint16_t*));
    for (uint32_t l = 0; l < m->layers; ++l) {
        size_t n = (size_t)m->layer[l].slots * m->kv_heads * m->head_dim;
        s->kcache[l] = (uint16_t*)calloc(n, 2);
        s->vcache[l] = (uint16_t*)calloc(n, 2);
    }
    size_t qd = (size_t)m->query_heads * m->head_dim, kvd = (size_t)m->kv_heads * m->head_dim;
    s->hidden = (float*)calloc(m->hidden, 4);
    s->normed = (float*)calloc(m->hidden, 4);
    s->q = (float*)calloc(qd, 4);
    s->k = (float*)calloc(kvd, 4);
    s->v = (float*)calloc(kvd, 4);
    s->att = (float*)calloc(qd, 4);
    s->out = (float*)calloc(m->hidden, 4);
    s->gate = (float*)calloc(m->ffn, 4);
    s->up = (float*)calloc(m->ffn, 4);
    s->act = (float*)calloc(m->ffn, 4);
    s->logits = (float*)calloc(m->vocab, 4);
    return s;
}

void or_state_destroy(or_state* s) {
    if (!s) return;
    for (uint32_t l = 0; l < s->m->layers; ++l) { free(s->kcache[l]); free(s->vcache[l]); }
    free(s->kcache); free(s->vcache);
    free(s->hidden); free(s->normed); free(s->q); free(s->k); free(s->v); free(s->att);
    free(s->out); free(s->gate); free(s->up); free(s->act); free(s->logits);
    free(s);
}

static void mm(const or_weight* w, const float* x, float* y, int threads) {
    or_matmul(w->type, w->piece, w->blocks, 0, w->rows, w->cols, x, 1, y, w->rows, threads);
}

/* One token's pass, as graph.cpp's Builder orders the launches (embed :155,
 * attention :159-230, gated_feed_forward :232-262, output :264-292); each
 * launch's arithmetic is batch-invariant (matmul.h "Determinism"), so a
 * token stepped alone has the bits it has in any step. */
static void forward_token(or_state* s, uint32_t id, uint32_t p, int threads) {
    const or_model* m = s->m;
    const uint32_t H = m->hidden, d = m->head_dim;
    float w32[32];
    /* gather.wgsl:25-53 */
    const uint32_t groups = H / 32;
    for (uint32_t g = 0; g < groups; ++g) {
        or_unpack(m->token_embd.type, m->token_embd.piece, m->token_embd.blocks, id * groups + g, w32);
        for (int j = 0; j < 32; ++j) s->hidden[g * 32 + j] = w32[j] * m->embed_scale;
    }
    s->pending_add = 0;
    s->pending_post = NULL;
    const float scale_log2e = (float)((double)m->attention_scale * 1.4426950408889634);
    for (uint32_t l = 0; l < m->layers; ++l) {
        const or_layer* L = &m->layer[l];
        or_norm_row(s->hidden, s->out, L->attn_norm, s->pending_post, H, m->epsilon, s->pending_add, s->normed);
        mm(&L->q, s->normed, s->q, threads);
        mm(&L->k, s->normed, s->k, threads);
        mm(&L->v, s->normed, s->v, threads);
        or_rope_shape rs = {d, m->query_heads, m->kv_heads, m->halves, L->q_norm != NULL, L->slots,
                            m->epsilon, L->turns, m->factors, L->q_norm, L->k_norm};
        or_rope_token(&rs, p, s->q, s->k, s->v, s->kcache[l], s->vcache[l]);
        or_attention_row(s->q, p, s->kcache[l], s->vcache[l], L->slots, L->window, scale_log2e, d,
                         m->query_heads, m->kv_heads, s->att);
        mm(&L->o, s->att, s->out, threads);
        s->pending_add = 1;
        s->pending_post = L->post_attn_norm;
        or_norm_row(s->hidden, s->out, L->ffn_norm, s->pending_post, H, m->epsilon, 1, s->normed);
        mm(&L->gate, s->normed, s->gate, threads);
        mm(&L->up, s->normed, s->up, threads);
        for (uint32_t j = 0; j < m->ffn; ++j) s->act[j] = or_activate(m->activation, s->gate[j]) * s->up[j];
        mm(&L->down, s->act, s->out, threads);
        s->pending_post = L->post_ffn_norm;
    }
}

int or_forward(or_state* s, const uint32_t* ids, uint32_t tokens, uint32_t position, int logits,
               const or_draw_settings* draw, float* logits_out, uint32_t* record, int threads) {
    const or_model* m = s->m;
    for (uint32_t t = 0; t < tokens; ++t) {
        if (ids[t] >= m->vocab) return -1;
        forward_token(s, ids[t], position + t, threads);
    }
    if (!logits) return 0;
    /* output (graph.cpp:264-292): final norm of the last row, head, top-k, draw */
    or_norm_row(s->hidden, s->out, m->output_norm, s->pending_post, m->hidden, m->epsilon, 1, s->normed);
    mm(&m->output, s->normed, s->logits, threads);
    if (logits_out) memcpy(logits_out, s->logits, (size_t)m->vocab * 4);
    uint32_t pairs[128];
    or_topk64(s->logits, m->vocab, pairs);
    or_draw_settings st = *draw;
    st.position = position;
    st.tokens = tokens;
    or_draw(pairs, &st, record);
    return 0;
}
