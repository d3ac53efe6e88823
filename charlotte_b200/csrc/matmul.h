// Arguments of the matrix-product kernels: the device form of the
// reference's `Matmul` constants struct (plainsight-systems/charlotte,
// src/core/kernels/matmul/matmul.wgsl:28-40: members[3] of {first word,
// blocks, first output row, rows}) plus the bindings it reads and writes.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace cb {

// What a product writes (matmul.h:594-599).
enum Epilogue : uint32_t { kWrite = 0, kQKV = 1, kGated = 2, kGatedByInput = 3 };

struct MemberArgs {
    const uint8_t* piece;   // the member's piece, 16-byte aligned, in the device layout
    uint32_t blocks;        // blocks in the piece (locates each stream)
    uint32_t first_row;     // first weight row read (a GLU half's first row)
    uint32_t rows;          // rows of the product this member gives
    uint32_t out_offset;    // Write: first output column; QKV: 0
};

struct MatmulArgs {
    uint32_t format;        // GGUF type: 2 Q4_0, 3 Q4_1, 8 Q8_0, 14 Q6_K, 30 BF16
    uint32_t columns;       // K, a multiple of 32
    uint32_t members;       // 1 to 3
    uint32_t total_rows;    // the members' rows together
    uint32_t epilogue;
    uint32_t activation;    // Gated and GatedByInput: 0 SiLU, 1 GELU tanh, 2 sigmoid
    uint32_t token;         // GatedByInput: the first token's row of u
    uint32_t tokens;        // rows of x (grid y)
    MemberArgs member[3];
    const float* x;         // [tokens][x_stride]
    uint32_t x_stride;
    float* out[3];          // [tokens][out_stride[m]]
    uint32_t out_stride[3];
    const float* gate_input;
    uint32_t gate_input_stride;
    uint32_t gate_input_column;
    unsigned int* fault;    // device word: a bounded wait that ran out sets a bit
    void* scratch;          // tensor form: x rounded to f16, [tokens][columns]
    uint64_t scratch_bytes; // tensor form: the dense form's split-K partials follow x16 when they fit
    const void* dense;      // tensor form: the weights as f16 in the dense layout (matmul_densify)
    const void* x16;        // dense form: x already f16 ([tokens][columns]), else rounded into scratch
    void* out16;            // dense form, gated: each output also f16 at [t·out_stride[0] + o]
    // Split form (matmul_split): range r's sum of product row p for token t
    // at range_sums[(r·tokens + t)·total_rows + p] (matmul.wgsl range_sum_at).
    float* range_sums;
    // One-token decode with the RMSNorm before the product folded in (the
    // decoder's own path; norm_gain NULL: x is read as given). Every CTA
    // computes norm_kernel's row — hidden (+ y, post-normed first when
    // norm_post_gain) — into its x stage; CTA 0 writes hidden + y to
    // norm_hidden_out (the residual stream's other buffer).
    const float* norm_hidden;
    const float* norm_y;
    const float* norm_post_gain;
    const float* norm_gain;
    float* norm_hidden_out;
    float norm_epsilon;
};

// Decode form over `tokens` rows of x (each token its own grid row): the
// reference's per-output order. PDL when `pdl`.
cudaError_t matmul_decode(const MatmulArgs& a, int sm_count, cudaStream_t stream, bool pdl);

// Tiled form over a step of `tokens` rows of x: the same sums, bit for bit,
// as a register-tiled GEMM on the CUDA cores. PDL when `pdl`.
cudaError_t matmul_tiled(const MatmulArgs& a, int sm_count, cudaStream_t stream, bool pdl);

// Split form (matmul.wgsl split_ranges :609 and combine_* :651-695): the
// tiled form's tiles once for each of the 32 ranges, each writing its range
// sums to a.range_sums, then a combine adding each output's 32 in order and
// applying the epilogue — the same bits as the other exact forms, with 32
// times the CTAs for products of few output tiles. Not for gated products.
cudaError_t matmul_split(const MatmulArgs& a, int sm_count, cudaStream_t stream, bool pdl);
// Whether the split form pays for a product: few output tiles for the SMs
// and ranges of at least two groups.
bool split_form(uint32_t tokens, uint32_t slots, uint32_t columns, uint32_t epilogue, int sm_count);

// Tensor-core form (tolerance tier, f16 operands, f32 accumulation in TMEM).
cudaError_t matmul_tensor(const MatmulArgs& a, cudaStream_t stream, bool pdl);
// The dense tensor form: the product's weights already decoded to f16 rows
// (matmul_densify, once), so both operands come by TMA; `sms` sizes the
// tiles and the split of K.
uint64_t matmul_dense_bytes(const MatmulArgs& a);
cudaError_t matmul_densify(const MatmulArgs& a, void* dense, cudaStream_t stream);
cudaError_t matmul_dense(const MatmulArgs& a, int sms, cudaStream_t stream, bool pdl);
uint64_t matmul_tensor_scratch_bytes(uint32_t tokens, uint32_t columns);

// Which exact form a step takes by default: the streamed (decode-layout)
// form's time grows with tokens × rows, the tiled GEMM's stays flat while
// its 128 × 128 tiles fit one wave, so the tiled form wins from a fixed
// amount of work (measured on B200, Qwen3 shapes: 4,096 rows from ~192
// tokens, 6,144 from ~128, 1,024 rows from 512–1,024 tokens). Its smallest
// tile is 32 tokens high, so steps of fewer tokens pay for 32: the
// vocabulary heads (150–260 K rows) stay streamed below ~24 tokens.
inline bool tiled_form(uint32_t tokens, uint32_t slots) {
    return tokens >= 24u && static_cast<uint64_t>(tokens) * slots >= 786432u;
}

// Shared memory the decode form needs at its smallest batch, for a width.
size_t matmul_decode_smem_bytes(uint32_t format, uint32_t columns);

}  // namespace cb
