// The fused decode step (decode_fused.cu): one persistent cooperative launch
// for the gather and every layer of a one-token step; its arguments.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "matmul.h"

namespace cb {

// A layer's products (tokens = 1, outputs bound to the step's buffers) and
// the rest of what its stages read.
struct FusedLayer {
    MatmulArgs qkv, o, gate_up, down;
    const float* attn_norm;
    const float* ffn_norm;
    const float* post_attn_norm;
    const float* post_ffn_norm;
    const float* q_norm;
    const float* k_norm;
    const float* turns;
    uint16_t* key_cache;
    uint16_t* value_cache;
    uint32_t window, slots;
};

struct FusedArgs {
    const FusedLayer* layers;   // device array
    uint32_t n_layers;
    uint32_t H, Hq, Hkv, d, ffn, halves;
    float epsilon, embed_scale, scale_log2e;
    const float* factors;       // llama3 rope factors or NULL
    const uint8_t* embed_piece;
    uint32_t embed_format, embed_blocks;
    const float* output_norm;
    float* hidden[2];           // the residual stream, ping-ponged at each add
    float* out;
    float* q;
    float* k;
    float* v;
    float* att;
    float* act;
    float* normed;              // the final norm's row, for the head
    float* partials;            // [chunks][Hq][d]
    float* stats;               // [chunks][Hq][2]
    const uint32_t* sampled;    // fed: the token is sampled[0]
    const uint32_t* ids;        // host-fed: ids[0]
    uint32_t fed;
    const uint32_t* state;      // state[0]: the step's position
    unsigned int* bar;          // 2 zeroed words: the grid barrier
    unsigned int* fault;
    uint32_t stage_bytes;       // a warp's ring slot
    uint32_t x_stage_floats;    // the CTA's x stage
};

struct FusedPlan {
    uint32_t warps, R, stage_bytes, x_stage_floats, ctas;
    size_t smem;
};

// Warps a CTA and rows a batch that fit shared memory for the widest
// product (max_columns; the largest row stage of a non-gated product, and of
// the gated one, whose batches are always two rows); warps == 0 when
// nothing fits.
FusedPlan fused_plan(uint32_t max_columns, uint32_t max_row_stage, uint32_t gated_row_stage, uint32_t head_dim,
                     int sm_count, int dev);

cudaError_t fused_step_run(const FusedArgs& a, const FusedPlan& plan, cudaStream_t stream);

}  // namespace cb
