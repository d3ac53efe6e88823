/*
 * charlotte_b200 — the C ABI of a B200 (sm_100a) CUDA backend for the hot
 * path of Charlotte (plainsight-systems/charlotte): GGUF dequant-matmul over
 * Q4_0 / Q8_0 / repacked Q6_K, RMSNorm, QK-norm + RoPE + KV append, chunked
 * attention over the f16 KV cache, embedding gather, top-k selection and the
 * draw. It stands where the reference's WebGPU dispatch layer
 * (src/core/kernels/program.{h,cpp}) and its WGSL kernels stand; the
 * reference's launchers, graph, KV-cache bookkeeping and loader are unchanged
 * callers.
 *
 * Conventions. Plain pointers and sizes only. Every buffer argument is a CUDA
 * device pointer unless its name says `host`. A `stream` is a cudaStream_t
 * (NULL: the legacy default stream). Weight pieces are in the reference's
 * device layout (src/core/formats/device_layout.h:121-136), each piece's
 * first byte 16-byte aligned and its length padded to 16. Every function
 * returns a cb_status; on failure cb_last_error() gives the calling thread's
 * message. Nothing here traps or spins without bound: a failed launch or an
 * invalid argument is a status, never a fault on purpose.
 */
#ifndef CHARLOTTE_B200_H
#define CHARLOTTE_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define CB_API __attribute__((visibility("default")))
#else
#define CB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* The five meanings of the reference's ProgramError
 * (src/core/kernels/program.h:71-77), plus argument errors. */
typedef enum cb_status {
    CB_OK = 0,
    CB_ERROR_BUILD = 1,        /* a program could not be built */
    CB_ERROR_STEP = 2,         /* a step (or a kernel call) failed to run */
    CB_ERROR_DEVICE_LOST = 3,  /* the CUDA context is no longer usable */
    CB_ERROR_CANCELLED = 4,    /* a step refused or abandoned unrun */
    CB_ERROR_INVALID = 5       /* an argument broke a stated precondition */
} cb_status;

/* GGUF tensor types a weight may take (src/core/gguf/types.h:41-43). */
enum { CB_F32 = 0, CB_F16 = 1, CB_Q4_0 = 2, CB_Q4_1 = 3, CB_Q8_0 = 8, CB_Q6_K = 14, CB_BF16 = 30 };

/* Copies the calling thread's last error message (NUL-terminated, truncated
 * to `capacity`); returns its full length. Replaces the message the
 * reference's callbacks carry (program.h:159-169). */
CB_API size_t cb_last_error(char* buffer, size_t capacity);

/* The library's version, "major.minor.patch". */
CB_API const char* cb_version(void);

/* The current device's streaming multiprocessor count (148 on a B200), or
 * a negative status. */
CB_API int cb_device_sm_count(void);

/* Reads and clears the current device's fault word: kernels whose bounded
 * waits ran out (a copy or a peer that never arrived) set bits in it instead
 * of spinning forever. Synchronizes the device. CB_OK when no bit was set;
 * otherwise CB_ERROR_STEP, with the bits in *faults (may be NULL). */
CB_API int cb_fault_check(unsigned int* faults);

/* A test hook for failure detection (no counterpart in the reference): on
 * the current device, the first wait of each kernel on a bulk copy (the
 * decode products and decode attention) gives up after `polls` polls (0:
 * at once, without polling) instead of the full bound, so a test can make a
 * wait run out — the kernel records the timeout in the fault word, drains
 * its copies (with the full bound) and returns — without any fault. A
 * negative value restores the full bound. Read by the kernels when they run
 * (captured graphs included); set it only between steps. Synchronous. */
CB_API int cb_debug_spin_limit(int32_t polls);

/* ---- matrix products --------------------------------------------------------
 * Replaces the matmul kernel's entry points decode_write, decode_qkv,
 * decode_gated, decode_gated_input (src/core/kernels/matmul/matmul.wgsl
 * :287-361) and the prefill forms (:520-695) behind matmul_launches
 * (src/core/kernels/matmul/matmul.h:672). One member is one weight piece;
 * a fused group (Q,K,V or gate,up) is two or three members, as the
 * reference's Matmul constants (matmul.wgsl:28-40) describe them. */
enum {
    CB_EPILOGUE_WRITE = 0,           /* y to out[0]                                  */
    CB_EPILOGUE_QKV = 1,             /* member m's rows to out[m]                     */
    CB_EPILOGUE_GATED = 2,           /* act(gate)·up to out[0]; members gate, up      */
    CB_EPILOGUE_GATED_BY_INPUT = 3   /* act(y)·u[t·stride + column + o] to out[0]     */
};
enum { CB_ACT_SILU = 0, CB_ACT_GELU_TANH = 1, CB_ACT_SIGMOID = 2 };

/* Flags of cb_matmul_run. */
enum {
    CB_MATMUL_PDL = 1u,      /* launch with programmatic dependent launch   */
    CB_MATMUL_TENSOR = 2u,   /* tokens > 1: the tcgen05 tensor-core form     */
    /* The exact forms give the same bits; these pick one (for benchmarks):
     * STREAMED decodes each weight once a pass of up to 16 tokens (decode
     * GEMV layout), TILED is the register-tiled GEMM. Default: by size. */
    CB_MATMUL_STREAMED = 4u,
    CB_MATMUL_TILED = 8u,
    /* The split form (split_ranges + combine, matmul.wgsl:609-695): the
     * tiled form's tiles once for each of the 32 ranges, each writing its
     * range sums to `scratch`, then a combine adding every output's 32 in
     * order — the same bits, 32 times the CTAs, for products of few output
     * tiles over a wide K. Not for gated products. Without the flag it is
     * chosen by size when `scratch` holds cb_matmul_split_bytes. */
    CB_MATMUL_SPLIT = 16u
};

typedef struct cb_member {
    const void* piece;     /* the weight piece (device layout), 16-B aligned          */
    uint32_t blocks;       /* blocks in the piece: locates each of its streams        */
    uint32_t first_row;    /* first weight row read (a GLU half's first row; else 0)  */
    uint32_t rows;         /* rows this member gives the product                      */
    uint32_t out_offset;   /* Write: first output column of its rows; otherwise 0     */
} cb_member;

typedef struct cb_matmul {
    uint32_t format;               /* CB_Q4_0, CB_Q4_1, CB_Q8_0, CB_Q6_K or CB_BF16      */
    uint32_t columns;              /* K, a multiple of 32                                */
    uint32_t members;              /* 1 to 3                                             */
    uint32_t epilogue;             /* CB_EPILOGUE_*                                      */
    uint32_t activation;           /* CB_ACT_*: GATED and GATED_BY_INPUT                 */
    cb_member member[3];
    const float* gate_input;       /* GATED_BY_INPUT's u, else NULL                      */
    uint32_t gate_input_stride;    /* floats between u's token rows                      */
    uint32_t gate_input_column;    /* u's first column                                   */
    uint32_t gate_input_token;     /* u's row of the first token                         */
    void* scratch;                 /* CB_MATMUL_TENSOR: cb_matmul_scratch_bytes() of
                                      device memory, 16-byte aligned (x rounded to f16);
                                      with `dense`, room after that lets the product
                                      split K (up to 8·tokens·slots floats); the exact
                                      forms take the split form's range sums here        */
    uint64_t scratch_bytes;
    const void* dense;             /* CB_MATMUL_TENSOR: NULL, or the product's weights
                                      as f16 rows written by cb_matmul_densify for these
                                      same members and epilogue (16-byte aligned): the
                                      dense form, both operands fed to the tensor cores
                                      by TMA; the pieces are then not read               */
    const void* x16;               /* with `dense`: NULL, or x already rounded to f16,
                                      [tokens][columns] (16-byte aligned) — read in place
                                      of rounding x (a norm's or a product's f16 copy)   */
    void* out16;                   /* with `dense`, GATED epilogue: NULL, or where each
                                      output is also written rounded to f16,
                                      [tokens][out_stride[0]] (the next product's x16)   */
} cb_matmul;

/* y[t][o] = Σ_k W[o][k]·x[t][k] for tokens t in [0, tokens), each output
 * added in the reference's order (matmul.h:34-50) unless CB_MATMUL_TENSOR.
 * x: [tokens][x_stride] f32. out[m]: [tokens][out_stride[m]] f32 (unused
 * entries may be NULL). */
CB_API int cb_matmul_run(const cb_matmul* m, const float* x, uint32_t x_stride, uint32_t tokens, float* const out[3],
                  const uint32_t out_stride[3], uint32_t flags, void* stream);
/* Scratch a product of `tokens` rows and `columns` K needs under `flags`
 * (0 for the exact forms). No counterpart in the reference (its prefill is
 * exact f32 only). */
CB_API uint64_t cb_matmul_scratch_bytes(uint32_t flags, uint32_t tokens, uint32_t columns);
/* The dense form's weights (no counterpart in the reference): each weight
 * of the product decoded exactly and rounded to f16 (nearest even), as
 * [slots][columns] rows — the members' rows in order; a gated product's in
 * 64-row units alternating gate and up rows of the same outputs, padded
 * with zero rows to whole 128-row pairs. A runtime writes them once (at
 * load) and passes them with every tensor-form call of the product. */
CB_API uint64_t cb_matmul_dense_bytes(const cb_matmul* m);
CB_API int cb_matmul_densify(const cb_matmul* m, void* dense, uint64_t dense_bytes, void* stream);
/* The split form's range-sum scratch for `tokens` rows of a product of
 * `rows` outputs: 32·tokens·rows floats, laid out as the reference's
 * range_sums (range_sum_at: (r·tokens + t)·rows + p, matmul.wgsl:600). */
CB_API uint64_t cb_matmul_split_bytes(uint32_t tokens, uint32_t rows);


/* ---- RMSNorm ------------------------------------------------------------------
 * Replaces norm.wgsl:80 behind norm_launch (src/core/kernels/norm/norm.h:220):
 * with `add`, hidden += y (y post-normed with post_gain first when given —
 * Gemma 3), the new hidden row written back; then normed = (x·r)·gain,
 * r = 1/sqrt(mean(x²) + epsilon), the sum of squares in the reference's
 * 256-way tree. `last_token`: the final norm, the step's last row only.
 * Rows up to 4096 wide, a multiple of 4. */
typedef struct cb_norm {
    float* hidden;            /* [tokens][width]                          */
    const float* output;      /* y, [tokens][width], with add             */
    const float* gain;        /* [width]; NULL: no gain (norm.h unit_gain) */
    const float* post_gain;   /* [width] or NULL                          */
    float* normed;            /* [tokens][width]                          */
    uint32_t width;
    uint32_t tokens;
    uint32_t add;
    uint32_t last_token;
    float epsilon;
    /* An encoder's variants (norm.h:69-82; zero leaves each off):
     * `scale`: one float multiplying x after the add (Gemma 4's layer output
     * scale; needs add); `add_only`: the add and x written back, nothing
     * normalized (needs add); `rows_per_token`: the launch covers tokens ×
     * rows_per_token rows, each normalized on its own (not with
     * last_token). */
    const float* scale;
    uint32_t add_only;
    uint32_t rows_per_token;
    /* NULL, or where normed is also written rounded to f16 (nearest even),
     * [rows][width]: a tensor-form product's x16. */
    void* normed16;
} cb_norm;
CB_API int cb_norm_run(const cb_norm* n, uint32_t flags, void* stream);

/* ---- QK-norm + RoPE + KV append -----------------------------------------------
 * Replaces rope.wgsl + rope_cache.wgsl behind rope_launch
 * (src/core/kernels/rope/rope.h:300): per token at position p = position +
 * row, query and key heads QK-normed (when gains are given) and turned by
 * p·θ_k (NEOX halves or adjacent pairs; llama3 factors divide the turns),
 * queries written back in place, keys and values packed f16 into cache slot
 * p mod slots ([slots][kv_heads][head_dim]). `turns` holds θ_k/2π rounded
 * once from f64 (rope.cpp:76; cb_rope_turns computes it). (Hq + 2·Hkv)·d/8
 * must be a multiple of 32; d is 64, 128 or 256. */
typedef struct cb_rope {
    float* query;
    float* key;                 /* read; written in place with `encode`    */
    float* value;               /* read; written in place with value_norm  */
    uint16_t* key_cache;
    uint16_t* value_cache;
    const float* query_gain;
    const float* key_gain;
    const float* factors;
    const float* turns;
    const uint32_t* position;   /* device word holding the step's position, or NULL */
    uint32_t position0;         /* the position when `position` is NULL            */
    uint32_t tokens;
    uint32_t head_dim;
    uint32_t query_heads;
    uint32_t kv_heads;
    uint32_t halves;
    uint32_t slots;
    float epsilon;
    /* Batched decode (no counterpart in the reference, which decodes one
     * sequence): nonzero makes row t the one token of sequence t, every row
     * at the step's position, its cache at key_cache/value_cache +
     * t·sequence_stride elements. Zero: rows are consecutive positions. */
    uint32_t rows_are_sequences;
    uint64_t sequence_stride;
    /* rope's encode form (rope_encode.wgsl, an encoder's): every head
     * written back in place, f32 — keys QK-normed and turned like queries —
     * and no cache (key_cache, value_cache, slots unused); with value_norm,
     * each value head also scaled by 1/sqrt(mean square + epsilon). This
     * form also takes heads of 512 (EmbeddingGemma 2's global layers). */
    uint32_t encode;
    uint32_t value_norm;
} cb_rope;
CB_API int cb_rope_run(const cb_rope* r, uint32_t flags, void* stream);
/* θ_k / 2π for k < d/2, base^(−2k/d) in f64 rounded once to f32 (host). */
CB_API void cb_rope_turns(double base, uint32_t head_dim, float* turns_host);

/* ---- attention ----------------------------------------------------------------
 * Replaces attention.wgsl main and combine behind attention_launches
 * (src/core/kernels/attention/attention.h:320): each query row at position
 * p attends keys p−window+1..p of the layer's f16 cache in 64-key chunks,
 * each chunk an online softmax in tiles of 2048/d keys, the chunks folded in
 * order — one launch, split over every chunk. `partials` holds
 * max_chunks·tokens·Hq·d floats, `stats` max_chunks·tokens·Hq·2, `tickets`
 * ceil(tokens/rows_per_tile)·Hkv zeroed words (left zero after each run);
 * max_chunks ≥ ceil((position + tokens)/64). scale_log2e = scale·log2(e). */
typedef struct cb_attention {
    const float* query;
    const uint16_t* key_cache;
    const uint16_t* value_cache;
    float* out;
    float* partials;
    float* stats;
    unsigned int* tickets;
    const uint32_t* position;
    uint32_t position0;
    uint32_t tokens;
    uint32_t head_dim;
    uint32_t query_heads;
    uint32_t kv_heads;
    uint32_t slots;
    uint32_t window;
    uint32_t max_chunks;
    float scale_log2e;
    /* Batched decode, as in cb_rope: row t is sequence t's query at the
     * step's position over its own cache (+ t·sequence_stride); `tickets`
     * then holds tokens·kv_heads zeroed words. */
    uint32_t rows_are_sequences;
    uint64_t sequence_stride;
    /* Decode shapes only (tokens == 1, or rows_are_sequences): when not NULL
     * (a host pointer, read at launch), this launch also does that rope step
     * for its rows, and no rope launch comes before it (no counterpart in the
     * reference, which launches rope then attention). `query` is then not
     * read: each CTA norms and turns its rows' raw queries from rope->query
     * in its prologue (they are not written back), and the CTA holding each
     * row's newest key turns that key, appends it and the value to the
     * caches, and stages both itself. Its fields must describe the same
     * rows, heads, caches and position as this struct's. */
    const cb_rope* rope;
    /* CB_RUN_TENSOR's form: NULL, or where out is also written rounded to
     * f16, [tokens][query_heads·head_dim] (the output product's x16). */
    void* out16;
} cb_attention;
CB_API int cb_attention_run(const cb_attention* a, uint32_t flags, void* stream);
/* Ticket words cb_attention needs for `tokens` rows. */
CB_API uint32_t cb_attention_tickets(uint32_t tokens, uint32_t query_heads, uint32_t kv_heads);

/* ---- block attention (an encoder's) -----------------------------------------------
 * Replaces block_attention.wgsl scores_of + weigh behind
 * block_attention_launches (src/core/kernels/block_attention/
 * block_attention.h:333): every row i of a step at position 0 attends the
 * step's own keys j with |i − j| ≤ half_window (the layer's window / 2),
 * f32 queries, keys and values as rope's encode form left them; the same
 * scores, maxima, weights and in-order sums, bit for bit, in one launch (no
 * scores buffer). tokens ≤ 1,024 at head_dim 512, head_dim a multiple of 64,
 * query_heads / kv_heads dividing 16. */
typedef struct cb_block_attention {
    const float* query;   /* [tokens][query_heads][head_dim] */
    const float* key;     /* [tokens][kv_heads][head_dim]    */
    const float* value;   /* [tokens][kv_heads][head_dim]    */
    float* out;           /* [tokens][query_heads][head_dim] */
    uint32_t tokens;
    uint32_t head_dim;
    uint32_t query_heads;
    uint32_t kv_heads;
    uint32_t half_window;
    float scale_log2e;
} cb_block_attention;
CB_API int cb_block_attention_run(const cb_block_attention* a, uint32_t flags, void* stream);

/* ---- pooling (an encoder's) -----------------------------------------------------
 * Replaces pool.wgsl mean and unit behind mean_launch and unit_launch
 * (src/core/kernels/pool/pool.h:107-121). MEAN: the mean of input rows
 * 0..tokens−1 ([tokens][width]), each column a chain of adds in row order
 * times 1/tokens, written at row tokens − 1 of output. UNIT: input's one row
 * over its Euclidean length into output (a zero row stays zero). width ≤
 * 4,096, a multiple of 4. */
enum { CB_POOL_MEAN = 0, CB_POOL_UNIT = 1 };
typedef struct cb_pool {
    const float* input;
    float* output;
    uint32_t width;
    uint32_t tokens;
    uint32_t kind;
} cb_pool;
CB_API int cb_pool_run(const cb_pool* p, uint32_t flags, void* stream);

/* ---- embedding gather -----------------------------------------------------------
 * Replaces gather.wgsl:25 behind gather_launches (src/core/kernels/gather/
 * gather.h:124): hidden[t] = unpack(table row of ids[t])·scale; a fed step
 * reads its one token from the last draw's record on the device. */
typedef struct cb_gather {
    const void* piece;
    uint32_t format;
    uint32_t blocks;
    uint32_t width;
    uint32_t first_row;
    uint32_t row_count;
    const uint32_t* ids;
    const uint32_t* sampled;
    uint32_t fed;
    uint32_t tokens;
    float scale;
    float* hidden;
    /* A fed step of several rows (batched decode): row t reads its token
     * from sampled[t·fed_stride]. Zero: one fed row, sampled[0]. */
    uint32_t fed_stride;
} cb_gather;
CB_API int cb_gather_run(const cb_gather* g, uint32_t flags, void* stream);

/* ---- top-k selection and the draw -------------------------------------------------
 * Replaces topk.wgsl first/merge and draw.wgsl behind topk_launches
 * (src/core/kernels/topk/topk.h:113) and sampler::draw_launch
 * (src/core/sampler/sampler.h:274): the 64 largest logits under the
 * reference's total order as (bits, token) candidates, then the draw
 * (temperature 0: candidate 0) into the 16-byte record {token, failed, u, 0}.
 * `partials` holds cb_select_tiles(count)·128 words, `ticket`
 * cb_select_tickets(count) zeroed words (left zero after each run).
 * count ≤ 262,144. */
typedef struct cb_select {
    const float* logits;
    uint32_t count;
    uint32_t* partials;
    unsigned int* ticket;
    uint32_t* candidates;       /* [64][2] */
    uint32_t* sampled;          /* [4]     */
    const uint32_t* position;
    uint32_t position0;
    uint32_t tokens;
    uint32_t seed0, seed1;
    uint32_t top_k;
    float temperature, top_p, min_p, log_min_p;
    /* Batched decode: `rows` independent selections (0 or 1: one), row r's
     * logits at logits + r·logits_stride, its partials, ticket words,
     * candidates and record at r times their one-row sizes; row r draws with
     * seed1 + r. */
    uint32_t rows;
    uint32_t logits_stride;
    /* A vocabulary split over ranks (no counterpart in the reference): the
     * logits are entries id_offset.. of the vocabulary (candidates carry
     * global ids); with candidates_only, the top 64 are written and no draw
     * is made (sampled may be NULL) — cb_select_merge_run finishes. */
    uint32_t id_offset;
    uint32_t candidates_only;
} cb_select;
CB_API int cb_select_run(const cb_select* s, uint32_t flags, void* stream);
CB_API uint32_t cb_select_tiles(uint32_t count);
CB_API uint32_t cb_select_tickets(uint32_t count);

/* cb_select_run for callers that cannot allocate device memory — a host
 * that plans every device byte up front against a budget, code where
 * cudaMalloc is not allowed or would stall the device, a plugin whose host
 * owns the allocator. No counterpart in the reference (its selection's
 * buffers are planned working buffers). Same inputs, outputs and results as
 * cb_select_run; `partials` and `ticket` must be NULL: the scratch is a
 * fixed 128 KiB array inside the library (every GPU that loads the library
 * holds it until the process exits), so count is at most 262,144. Allocates
 * nothing. The first call on a device looks up the array's address (make it
 * before any stream capture). All calls share the array: calls that overlap
 * on the GPU race — order them on one stream. */
CB_API int cb_select_run_static(const cb_select* s, uint32_t flags, void* stream);

/* The merge of a vocabulary split (no counterpart in the reference): each
 * row's `lists` candidate lists, list l of row r at pairs
 * ((l·rows + r)·64 ...) of lists_data — what an all-gather of every rank's
 * candidates_only output gives — merged into the row's top 64 under the
 * same total order (the union holds the whole vocabulary's top 64, so the
 * result is one selection's over the whole vocabulary), then the draw,
 * rows' records at sampled + 4·r and candidates at candidates + 128·r. */
typedef struct cb_select_merge {
    const uint32_t* lists_data;
    uint32_t lists;             /* 1 to 64 (ranks)                           */
    uint32_t rows;
    uint32_t* candidates;       /* [rows][64][2]                             */
    uint32_t* sampled;          /* [rows][4]                                 */
    const uint32_t* position;
    uint32_t position0;
    uint32_t tokens;
    uint32_t seed0, seed1;
    uint32_t top_k;
    float temperature, top_p, min_p, log_min_p;
} cb_select_merge;
CB_API int cb_select_merge_run(const cb_select_merge* m, uint32_t flags, void* stream);

/* Flags of the kernel entry points above. CB_RUN_TENSOR (cb_attention_run
 * only): steps of 16 positions or more (not rows_are_sequences, no fused rope)
 * with head dimension 64 or 128 and 1, 2, 4 or 8 query heads a kv head run
 * on the tensor cores — f16 queries and weights, f32 sums in the tensor
 * cores' order: the tolerance tier, not the reference's bits (no counterpart
 * in the reference); other shapes keep the exact form. */
enum { CB_RUN_PDL = 1u, CB_RUN_TENSOR = 2u };

/* ---- weight layout ------------------------------------------------------------
 * The device layout of a weight piece (src/core/formats/device_layout.h:
 * 121-136; Q6_K repacked as src/core/formats/q6_k/q6_k.h:9-21 describes),
 * made on the host from the file's stored blocks — what the reference's
 * PieceWriter writes (src/core/residency/piece_writer.h). `piece_host`
 * holds cb_piece_bytes(format, blocks) bytes (the stored size rounded up to
 * 16). */
CB_API size_t cb_piece_bytes(uint32_t format, uint64_t blocks);
CB_API int cb_piece_from_stored(uint32_t format, const void* stored_host, uint64_t blocks, void* piece_host);

/* ---- a whole decoder ------------------------------------------------------------
 * The pass the reference's graph builds (src/core/graph/graph.cpp: embed,
 * per layer attention then gated feed-forward, output) for Qwen3, Llama 3
 * and Gemma 3 shaped models, run on the CUDA kernels above: weights uploaded
 * once, an f16 KV cache per layer (a ring of window + step slots for a
 * sliding-window layer), each step's launches in the reference's order, a
 * decode step captured once as a CUDA graph and replayed (its position and
 * fed token read on the device). Stands in for Program + Upload
 * (src/core/kernels/program.h:262-331, residency/upload.h) for a caller that
 * brings its weights as host memory. */
typedef struct cb_weight {
    uint32_t format;             /* CB_Q4_0, Q4_1, Q8_0, Q6_K, BF16 (matmuls); rows=0: absent */
    uint32_t rows, cols;         /* rows of cols weights (cols a multiple of the block) */
    const void* stored_host;     /* the file's stored blocks                        */
} cb_weight;

typedef struct cb_layer_weights {
    const float* attn_norm;      /* [hidden]                                       */
    cb_weight q, k, v, o;
    const float* q_norm;         /* [head_dim] or NULL (no QK-norm)                */
    const float* k_norm;
    const float* post_attn_norm; /* [hidden] or NULL (Gemma 3's post-norms)        */
    const float* ffn_norm;
    cb_weight gate, up, down;
    const float* post_ffn_norm;
    uint32_t window;             /* keys a query reads: the context for a global layer */
    float rope_base;
} cb_layer_weights;

typedef struct cb_model {
    uint32_t layers, hidden, query_heads, kv_heads, head_dim, ffn, vocab, context;
    float epsilon, attention_scale, embed_scale;
    uint32_t halves;             /* 1 NEOX (Qwen3, Gemma 3), 0 adjacent (Llama)   */
    uint32_t activation;         /* CB_ACT_SILU or CB_ACT_GELU_TANH                */
    const float* rope_factors;   /* [head_dim/2] or NULL (llama3 rope_freqs)      */
    cb_weight token_embd;
    const float* output_norm;
    cb_weight output;            /* rows = 0: tied to token_embd                   */
    const cb_layer_weights* layer;
} cb_model;

/* The draw's settings (policy::SamplingSettings through sampler::apply into
 * the Step, src/core/kernels/interface.h:165-192). temperature 0: greedy. */
typedef struct cb_sampling {
    uint32_t seed0, seed1;
    uint32_t top_k;
    float temperature, top_p, min_p;
} cb_sampling;

typedef struct cb_decoder cb_decoder;

enum {
    /* Steps of 128 tokens or more run their products (CB_MATMUL_TENSOR)
     * and, where it fits, their attention (CB_RUN_TENSOR) in the
     * tensor-core forms, the tolerance tier, instead of the exact forms;
     * shorter steps (decode) and the head's last-token product stay exact.
     * No counterpart in the reference. */
    CB_DECODER_TENSOR_PREFILL = 1u
};

/* Uploads the model and allocates its caches and working buffers for steps
 * of up to max_step_tokens (the reference's prefill block is 512). */
CB_API int cb_decoder_create(const cb_model* m, uint32_t max_step_tokens, uint32_t flags, cb_decoder** out);
CB_API void cb_decoder_destroy(cb_decoder* d);

/* One step (Program::run(Step)): `tokens` ids from host memory at
 * `position`; with `logits`, the last token's head, top-k and draw, its
 * 16-byte record {token, failed, u, 0} copied to record_host. Synchronous. */
CB_API int cb_decoder_step(cb_decoder* d, const uint32_t* ids_host, uint32_t tokens, uint32_t position,
                           uint32_t logits, const cb_sampling* s, uint32_t* record_host);

/* `steps` fed decode steps after the last step (each reads the last draw's
 * token on the device), from one CUDA graph replayed back to back; the
 * drawn tokens (and each step's failed flag) copied to tokens_host. With
 * device_ms, the replays' device time (CUDA events around them). */
CB_API int cb_decoder_generate(cb_decoder* d, uint32_t steps, const cb_sampling* s, uint32_t* tokens_host,
                               uint32_t* failed_host, float* device_ms);

/* The last step's logits [vocab] to host memory. */
CB_API int cb_decoder_logits(cb_decoder* d, float* logits_host);

/* ---- batched decode (no counterpart in the reference, which runs one
 * sequence): a decoder holding `sequences` independent sequences, each with
 * its own KV caches. A prompt goes in per sequence (cb_decoder_step_sequence:
 * consecutive positions of sequence `seq`, its draw in record row `seq`);
 * then every sequence steps together, one token each at one common position
 * — cb_decoder_step_batch from host ids, or cb_decoder_generate (fed from
 * each row's last draw; tokens_host then holds steps × sequences ids, step
 * by step). A row's arithmetic is that of its sequence decoded alone, so
 * its tokens and logits are bit-identical to a one-sequence decoder's. */
CB_API int cb_decoder_create_batch(const cb_model* m, uint32_t max_step_tokens, uint32_t sequences, uint32_t flags,
                                   cb_decoder** out);
CB_API int cb_decoder_step_sequence(cb_decoder* d, uint32_t seq, const uint32_t* ids_host, uint32_t tokens,
                                    uint32_t position, uint32_t logits, const cb_sampling* s, uint32_t* record_host);
/* One token of every sequence (ids_host[sequences]) at `position`; the
 * records [sequences][4] to records_host. Synchronous. */
CB_API int cb_decoder_step_batch(cb_decoder* d, const uint32_t* ids_host, uint32_t position, const cb_sampling* s,
                                 uint32_t* records_host);
/* Row `row`'s logits of the last step [vocab] to host memory. */
CB_API int cb_decoder_logits_row(cb_decoder* d, uint32_t row, float* logits_host);

/* A vocabulary split over ranks (no counterpart in the reference): a
 * batched step up to the final norm (ids_host NULL: each row fed from its
 * record in cb_decoder_device_sampled), leaving the normed rows
 * [sequences][hidden] at cb_decoder_device_normed on cb_decoder_stream;
 * the caller runs its head shard (cb_decoder_head gives the weight; its
 * member's first_row and rows select the shard), cb_select_run with
 * candidates_only, the exchange, and cb_select_merge_run, and writes each
 * of its rows' record back into cb_decoder_device_sampled for the next
 * step. Returns after the enqueued work completes. */
CB_API int cb_decoder_step_body(cb_decoder* d, const uint32_t* ids_host, uint32_t position);
CB_API void* cb_decoder_stream(cb_decoder* d);
CB_API const float* cb_decoder_device_normed(cb_decoder* d);
CB_API uint32_t* cb_decoder_device_sampled(cb_decoder* d);
CB_API int cb_decoder_head(cb_decoder* d, cb_member* head, uint32_t* format, uint32_t* columns);

/* Device pointers of the decoder's working buffers, for callers that feed
 * it from their own kernels: the logits [vocab] and the sampled record [4]. */
CB_API const float* cb_decoder_device_logits(cb_decoder* d);

/* ---- buffers and programs: the reference's Upload and Program over CUDA ----------
 * The reference's kernel launchers describe every launch of a graph as a
 * kernels::Launch (src/core/kernels/interface.h:318-365) over the buffers a
 * residency plan names; kernels::Program (src/core/kernels/program.h:262-331)
 * builds them once at load and runs them a step at a time. These entry points
 * are that Program over CUDA: cb_buffers holds the plan's buffers (what
 * residency::Upload holds, src/core/residency/upload.h:245-332), cb_launch
 * is a Launch in plain C, cb_step is the reference's Step byte for byte, and
 * cb_program builds the launches onto this library's kernels and runs steps
 * without blocking — at most two outstanding, each one's readback delivered
 * to its callback in the order the steps were run (program.h:62-70,
 * src/core/kernels/order.h:30). */

typedef struct cb_buffers cb_buffers;
/* `count` zeroed device buffers of `sizes` bytes (each 256-byte aligned). */
CB_API int cb_buffers_create(const uint64_t* sizes, uint32_t count, cb_buffers** out);
CB_API void cb_buffers_destroy(cb_buffers* b);
/* Host bytes into / out of buffer `buffer` at `offset` (synchronous). */
CB_API int cb_buffers_write(cb_buffers* b, uint32_t buffer, uint64_t offset, const void* host, uint64_t bytes);
CB_API int cb_buffers_read(cb_buffers* b, uint32_t buffer, uint64_t offset, void* host, uint64_t bytes);
/* The device address of a buffer, or NULL. */
CB_API void* cb_buffers_device(const cb_buffers* b, uint32_t buffer);

/* The kernels a launch names (the reference's WGSL modules, by the shaders
 * its launchers embed: shaders::matmul, norm, rope + rope_cache, attention,
 * gather, topk, draw). */
enum {
    CB_KERNEL_UNKNOWN = 0,
    CB_KERNEL_MATMUL = 1,
    CB_KERNEL_NORM = 2,
    CB_KERNEL_ROPE_CACHE = 3,
    CB_KERNEL_ATTENTION = 4,
    CB_KERNEL_GATHER = 5,
    CB_KERNEL_TOPK = 6,
    CB_KERNEL_DRAW = 7,
    CB_KERNEL_ROPE_ENCODE = 8,       /* rope.wgsl + rope_encode.wgsl (an encoder's)  */
    CB_KERNEL_BLOCK_ATTENTION = 9,   /* block_attention.wgsl (scores_of, weigh)      */
    CB_KERNEL_POOL = 10              /* pool.wgsl (mean, unit)                       */
};
enum { CB_ROWS_EVERY_TOKEN = 0, CB_ROWS_LAST_TOKEN = 1 };            /* interface.h Rows      */
enum { CB_KEY_SPLIT_NONE = 0, CB_KEY_SPLIT_PER_CHUNK = 1, CB_KEY_SPLIT_WHEN_SPLIT = 2 };   /* KeySplit */
enum { CB_NO_FORMAT = 0xFFFFFFFFu };

/* interface.h Binding: a range of a planned buffer. */
typedef struct cb_binding {
    uint32_t buffer;
    uint32_t reserved;
    uint64_t offset;
    uint64_t size;
} cb_binding;

/* interface.h Override. */
typedef struct cb_override {
    const char* name;   /* NUL-terminated */
    double value;
} cb_override;

/* interface.h Launch, field for field. */
typedef struct cb_launch {
    uint32_t kernel;               /* CB_KERNEL_*                                      */
    const char* entry_point;       /* NUL-terminated                                   */
    uint32_t format;               /* GGUF type of the format it unpacks, or CB_NO_FORMAT */
    uint32_t pack_format;          /* GGUF type of the format it packs, or CB_NO_FORMAT */
    const uint8_t* constants;      /* binding 1's bytes                                */
    uint32_t constants_bytes;
    const cb_binding* bindings;    /* bindings 2 onward                                */
    uint32_t binding_count;
    uint32_t invocations_per_row;
    uint32_t workgroup_size;
    uint32_t rows;                 /* CB_ROWS_*                                        */
    const cb_override* overrides;
    uint32_t override_count;
    uint32_t rows_per_tile;
    uint32_t key_split;            /* CB_KEY_SPLIT_*                                   */
    uint32_t window;
    uint32_t partial_rows;
    uint32_t tokens_least, tokens_most;   /* TokenRange                                */
    uint32_t row_divisor;
} cb_launch;

/* interface.h Step (64-byte head, then the identifiers), byte for byte. */
typedef struct cb_step {
    uint32_t position, tokens, logits, fed;
    uint32_t seed[2];
    uint32_t top_k;
    float temperature, top_p, min_p, log_min_p;
    uint32_t columns, media, media_token, padding1, padding2;
    uint32_t ids[512];
} cb_step;

/* A step's end (program.h StepCallback): its status and message (empty on
 * success), and its copy of the readback range (NULL for a step that read
 * none or failed); valid during the call only. */
typedef void (*cb_step_callback)(int status, const char* message, const void* readback, uint64_t readback_bytes,
                                 void* userdata);
/* A profiled step's end (program.h ProfileCallback): as cb_step_callback,
 * plus the step's device time: its begin and end, and the end of each launch
 * it ran, in nanoseconds from its begin, by the launch's index in the graph. */
typedef void (*cb_profile_callback)(int status, const char* message, const void* readback, uint64_t readback_bytes,
                                    uint64_t begin_ns, uint64_t end_ns, const uint32_t* launch_index,
                                    const uint64_t* launch_end_ns, uint32_t launches_timed, void* userdata);

typedef struct cb_program cb_program;
/* Program::build: the launches in the graph's order over `buffers`
 * (borrowed: they outlive the program), reading back `readback` (NULL: none)
 * from each step that asks for logits. A launch of a kernel, entry point,
 * format or variant this backend has no form for is refused, CB_ERROR_BUILD,
 * with its index and what it names. */
CB_API int cb_program_build(cb_buffers* buffers, const cb_launch* launches, uint32_t count, const cb_binding* readback,
                            cb_program** out);
/* Program::run: enqueues one step and returns; `done` fires from
 * cb_program_poll once it has finished, in run order. A step past position
 * 2^24 fails unrun (CB_ERROR_STEP); a third while two are outstanding is
 * refused at once, its callback fired before this returns. */
CB_API int cb_program_run(cb_program* p, const cb_step* step, cb_step_callback done, void* userdata);
/* Program::run_profiled: the first `launches` launches of the step, each
 * timed by CUDA events on the program's stream; not beside unprofiled steps. */
CB_API int cb_program_run_profiled(cb_program* p, const cb_step* step, uint32_t launches, cb_profile_callback done,
                                   void* userdata);
/* Fires the callbacks of finished steps, oldest first; with `wait`, first
 * blocks until the oldest outstanding step has finished (so a caller that
 * keeps two steps in flight waits for one, runs the next, and so on).
 * Returns the callbacks fired. */
CB_API int cb_program_poll(cb_program* p, uint32_t wait);
CB_API uint32_t cb_program_outstanding(const cb_program* p);
CB_API uint32_t cb_program_launch_count(const cb_program* p);
/* The CUDA stream the program's steps run on. */
CB_API void* cb_program_stream(const cb_program* p);
/* Destroys the program: steps still outstanding fire CB_ERROR_CANCELLED. */
CB_API void cb_program_destroy(cb_program* p);

#ifdef __cplusplus
}
#endif
#endif
