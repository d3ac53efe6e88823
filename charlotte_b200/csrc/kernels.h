// The non-matmul kernels of the hot path. Their arguments are the public C
// structs (include/charlotte_b200.h), each the device form of a reference
// launcher's constants and bindings (plainsight-systems/charlotte,
// src/core/kernels/<op>/<op>.h).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "charlotte_b200.h"

namespace cb {

using NormArgs = cb_norm;
using RopeArgs = cb_rope;
using AttentionArgs = cb_attention;
using GatherArgs = cb_gather;
using SelectArgs = cb_select;

cudaError_t norm_run(const NormArgs& a, cudaStream_t stream, bool pdl);
cudaError_t rope_run(const RopeArgs& a, cudaStream_t stream, bool pdl);
cudaError_t attention_run(const AttentionArgs& a, cudaStream_t stream, bool pdl);
uint32_t attention_row_tiles(uint32_t tokens, uint32_t query_heads, uint32_t kv_heads, bool sequences);
// The many-query form (attention_prefill.cu): same bits, a CTA per query tile.
bool attention_prefill_fits(const AttentionArgs& a);
cudaError_t attention_prefill_run(const AttentionArgs& a, cudaStream_t stream, bool pdl);
// The tensor-core form (attention_tensor.cu), the tolerance tier: steps of
// 16 positions or more, head dimensions 64 and 128, 1, 2, 4 or 8 query heads a kv head.
bool attention_tensor_fits(const AttentionArgs& a);
cudaError_t attention_tensor_run(const AttentionArgs& a, cudaStream_t stream, bool pdl);
// Steps of at least this many rows take the many-query form.
constexpr uint32_t kPrefillAttentionRows = 32;
cudaError_t gather_run(const GatherArgs& a, cudaStream_t stream, bool pdl);
// An encoder's (encoder.cu): block attention and pooling.
bool block_attention_fits(const cb_block_attention& a);
cudaError_t block_attention_run(const cb_block_attention& a, cudaStream_t stream, bool pdl);
cudaError_t pool_run(const cb_pool& p, cudaStream_t stream, bool pdl);
cudaError_t select_merge_run(const cb_select_merge& a, cudaStream_t stream, bool pdl);
cudaError_t select_run(const SelectArgs& a, cudaStream_t stream, bool pdl);
uint32_t select_tiles(uint32_t count);

}  // namespace cb
