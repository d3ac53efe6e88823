/*
 * CPU oracle for the charlotte_b200 hot path — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the arithmetic Charlotte's WGSL kernels perform on
 * its hot path (GGUF dequant-matmul, RMSNorm, QK-norm + RoPE + KV append,
 * chunked online-softmax attention, embedding gather, top-k selection and the
 * draw), in the reference's order of operations. Only the tests, the smoke
 * check and bench.py's CPU-baseline leg load it, and only as the checker or the
 * timed CPU baseline; the product (libcharlotte_b200.so) never links or calls
 * anything here.
 *
 * Where WGSL leaves a result to the implementation (the contraction of a*b+c,
 * the built-ins dot, inverseSqrt, exp2, cos, sin, ldexp) this file fixes one
 * definition, and the CUDA kernels implement the same definition, so the two
 * agree bit for bit:
 *   dot4(a,b)       fmaf(a3,b3, fmaf(a2,b2, fmaf(a1,b1, a0*b0)))
 *   inverseSqrt(v)  1.0f / sqrtf(v)          (two correctly rounded ops)
 *   x*y + z*w       fmaf(x, y, z*w)          (attention folds, rotations)
 *   acc += p*v      fmaf(p, v, acc)
 *   exp2, exp, cos, sin: the published methods named at or_exp2, or_sincos.
 *   ldexp(p, k)     p * 2^k by exact power-of-two multiplies (or_scale2)
 * Everything is compiled without contraction (-ffp-contract=off) so that
 * only the explicit fmaf calls fuse.
 *
 * Parity is pinned: the dequantizers and the Q6_K repack are checked against
 * the reference's own C++ (the tests/support dequantizer headers and
 * src/core/formats/q6_k/q6_k_repack.cpp, compiled from its sources into
 * oracle/_ref), and against its known-answer tests (tests/quant_q4_0_test.cpp,
 * tests/sampler_test.cpp Philox vectors) — see tests/test_oracle_pins.py.
 */
#ifndef CHARLOTTE_ORACLE_H
#define CHARLOTTE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGUF tensor types (src/core/gguf/types.h:41-43). */
enum { OR_F32 = 0, OR_F16 = 1, OR_Q4_0 = 2, OR_Q4_1 = 3, OR_Q8_0 = 8, OR_Q6_K = 14, OR_BF16 = 30 };

/* Activations (matmul.wgsl:189-205 `activation` override). */
enum { OR_SILU = 0, OR_GELU_TANH = 1, OR_SIGMOID = 2 };

/* ---- scalar numerics ---------------------------------------------------- */
float or_fp16_to_fp32(uint16_t h);          /* src/core/quant/q4_0.h:66 */
uint16_t or_fp32_to_fp16_sat(float f);      /* formats/f16/f16_pack.wgsl:9-15 */
float or_exp_nonpositive(float x);          /* matmul.wgsl:169-182 */
float or_activate(int activation, float g); /* matmul.wgsl:189-205 */
float or_exp2(float x);                     /* attention.wgsl's exp2, x <= 0 */
void or_sincos(float angle, float* s, float* c);
float or_scale2(float p, int k);
float or_dot4(const float* a, const float* b);

/* ---- formats ------------------------------------------------------------- */
/* Bytes of one stored block, and weights in it. */
uint32_t or_block_bytes(int type);
uint32_t or_block_weights(int type);
/* Dequantize stored (file-order, AoS) blocks in ggml's order of operations
 * (tests/support/q4_0_reference.h:25, q8_0_reference.h:15, q6_k_reference.h:17). */
int or_dequant_stored(int type, const uint8_t* data, size_t blocks, float* out);
/* Device piece size: the stored bytes rounded up to 16 (plan.h binds at 4;
 * the CUDA backend pads pieces to 16 so every stream starts 16-B aligned). */
size_t or_piece_bytes(int type, size_t blocks);
/* Stored blocks -> the device layout's streams (device_layout.h:121-136),
 * Q6_K repacked as q6_k.h:9-21 describes. */
int or_to_piece(int type, const uint8_t* stored, size_t blocks, uint8_t* piece);
/* The 32 weights of `group` of a piece (each format's unpack(), e.g.
 * q4_0.wgsl:6, q8_0.wgsl:6, q6_k.wgsl:13). */
int or_unpack(int type, const uint8_t* piece, uint32_t blocks_in_piece, uint32_t group, float* out32);

/* ---- matrix products (matmul.wgsl) ---------------------------------------- */
/* y[t*y_stride + o] for rows o in [0, rows) of a piece whose rows are K wide,
 * tokens t in [0, tokens) of x (row stride K): each output the 32 range sums
 * of decode_ranges/tile_range added in order (matmul.h:34-50). */
int or_matmul(int type, const uint8_t* piece, uint32_t blocks_in_piece, uint32_t row0, uint32_t rows,
              uint32_t K, const float* x, uint32_t tokens, float* y, uint32_t y_stride, int threads);

/* ---- norm (norm.wgsl:80) --------------------------------------------------- */
/* One row: optional add of `output` (post-normed first when post_gain), the
 * new hidden row written back, then normed = (x*r)*gain. width <= 4096. */
void or_norm_row(float* hidden, const float* output, const float* gain, const float* post_gain,
                 uint32_t width, float epsilon, int add, float* normed);

/* ---- rope cache form (rope.wgsl + rope_cache.wgsl) ------------------------ */
typedef struct or_rope_shape {
    uint32_t head_dim, query_heads, kv_heads;
    int halves;       /* 1 NEOX (Halves), 0 NORM (Adjacent) */
    int qk_norm;
    uint32_t slots;
    float epsilon;
    const float* turns;   /* d/2 floats: theta_k / 2pi rounded once (rope.cpp:76) */
    const float* factors; /* d/2 floats or NULL (llama3 rope_freqs) */
    const float* query_gain, *key_gain;  /* d floats each, when qk_norm */
} or_rope_shape;
/* One token at position p: q [Hq*d] in place; k,v [Hkv*d] -> f16 caches. */
void or_rope_token(const or_rope_shape* s, uint32_t p, float* q, const float* k, const float* v,
                   uint16_t* key_cache, uint16_t* value_cache);
void or_rope_turns(double base, uint32_t head_dim, float* turns);

/* ---- attention (attention.wgsl:138,363) ----------------------------------- */
/* One query row at position p over the layer's f16 cache: out [Hq*d]. */
void or_attention_row(const float* q, uint32_t p, const uint16_t* key_cache, const uint16_t* value_cache,
                      uint32_t slots, uint32_t window, float scale_log2e, uint32_t head_dim,
                      uint32_t query_heads, uint32_t kv_heads, float* out);

/* ---- an encoder's kernels (graph/encoder.h) -------------------------------- */
/* norm.wgsl:80-198 with the encoder's variants for one row: the add (y
 * post-normed first with post_gain, times post_scale), x = (x + y)·scale[0]
 * when `scale`, the new hidden row written back; without `normalize` nothing
 * more; else normed = (x·r)·gain, or x·r when gain is NULL. */
void or_norm_row_ex(float* hidden, const float* output, const float* gain, const float* post_gain, float post_scale,
                    const float* scale, uint32_t width, float epsilon, int add, int normalize, float* normed);
/* rope_encode.wgsl for one token at position p, in place: query and key
 * heads QK-normed (qk_norm) and turned, value heads normalized without a
 * gain when value_norm; no cache. */
void or_rope_encode_token(const or_rope_shape* s, uint32_t p, int value_norm, float* q, float* k, float* v);
/* block_attention.wgsl scores_of + weigh for the whole step of n rows:
 * q [n][hq][d], k and v [n][hkv][d], out [n][hq][d]; key j live for row i
 * when |i - j| <= half_window. */
void or_block_attention(const float* q, const float* k, const float* v, uint32_t n, uint32_t d, uint32_t query_heads,
                        uint32_t kv_heads, uint32_t half_window, float scale_log2e, float* out);
/* pool.wgsl mean: the mean of n rows of `width` (a chain of adds a column in
 * row order, times 1/n); unit: a row over its Euclidean length (zeros stay
 * zeros). */
void or_pool_mean(const float* rows, uint32_t n, uint32_t width, float* mean);
void or_pool_unit(const float* row, uint32_t width, float* unit);

/* ---- selection and draw (topk.wgsl, draw.wgsl) ----------------------------- */
uint32_t or_key_of(uint32_t bits);   /* topk.wgsl:28 */
uint32_t or_bits_of(uint32_t key);   /* topk.wgsl:43 */
/* Top-64 (logit desc, token asc) as (bits, id) pairs; padded with
 * (0xFFFFFFFF, 0xFFFFFFFF) when count < 64. */
void or_topk64(const float* logits, uint32_t count, uint32_t* pairs128);
void or_philox4x32_10(const uint32_t counter[4], const uint32_t key[2], uint32_t out[4]);
typedef struct or_draw_settings {
    uint32_t position, tokens, seed0, seed1, top_k;
    float temperature, top_p, min_p, log_min_p;
} or_draw_settings;
/* The sampled record {token, failed, u bits, 0} from 64 candidates. */
void or_draw(const uint32_t* pairs128, const or_draw_settings* s, uint32_t* record4);

/* ---- whole decoder pass (graph.cpp: embed, attention, gated_feed_forward, output) */
typedef struct or_weight {
    int type;
    const uint8_t* piece;      /* device layout */
    uint32_t blocks;           /* blocks in the piece */
    uint32_t rows, cols;
} or_weight;

typedef struct or_layer {
    const float* attn_norm;
    or_weight q, k, v, o;
    const float* q_norm, *k_norm;      /* NULL without QK-norm */
    const float* post_attn_norm;       /* Gemma 3, else NULL */
    const float* ffn_norm;
    or_weight gate, up, down;
    const float* post_ffn_norm;        /* Gemma 3, else NULL */
    uint32_t window;                   /* attention window (context for global) */
    uint32_t slots;                    /* cache slots */
    const float* turns;                /* d/2 */
} or_layer;

typedef struct or_model {
    uint32_t layers, hidden, query_heads, kv_heads, head_dim, ffn, vocab;
    float epsilon, attention_scale, embed_scale;
    int halves, activation;
    const float* factors;              /* NULL or d/2 */
    or_weight token_embd;
    const float* output_norm;
    or_weight output;                  /* head (may be token_embd's bytes) */
    const or_layer* layer;
} or_model;

typedef struct or_state or_state;
or_state* or_state_create(const or_model* m);
void or_state_destroy(or_state* s);
/* Runs `tokens` token ids from `position`; when `logits`, writes the last
 * token's logits [vocab] (may be NULL) and its 16-byte sampled record. */
int or_forward(or_state* s, const uint32_t* ids, uint32_t tokens, uint32_t position, int logits,
               const or_draw_settings* draw, float* logits_out, uint32_t* record4, int threads);

#ifdef __cplusplus
}
#endif
#endif
