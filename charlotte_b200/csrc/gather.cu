// Token-embedding gather (plainsight-systems/charlotte,
// src/core/kernels/gather/gather.wgsl:25-53; launcher gather.h:124): each of
// the step's rows takes its token's row of the table, decoded 32 weights at
// a time through the format's unpack, times the scale (√width for Gemma 3,
// 1 otherwise). A fed step's one token is the last draw's (sampled[0]),
// read on the device, so decode never waits on the host. A token outside
// this piece's rows is another piece's launch's to write.
#include <cuda_runtime.h>

#include <cstdint>

#include "formats.cuh"
#include "kernels.h"
#include "tma.cuh"

namespace cb {

namespace {

template <typename F, int k>
__device__ __forceinline__ void put(const F& f, const typename F::Consts& c, float scale, float* out) {
    out[k] = F::template weight<k>(f, c) * scale;
}

template <typename F, int... ks>
__device__ __forceinline__ void put_all(const F& f, float scale, float* out, std::integer_sequence<int, ks...>) {
    const typename F::Consts c = f.consts();
    (put<F, ks>(f, c, scale, out), ...);
}

template <typename F>
__global__ void gather_kernel(GatherArgs a) {
    grid_dependency_wait();
    const uint32_t groups = a.width / 32u;
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t row = i / groups, g = i % groups;
    if (row >= a.tokens) return;
    const uint32_t token = a.fed ? a.sampled[static_cast<size_t>(row) * a.fed_stride] : a.ids[row];
    if (token < a.first_row || token - a.first_row >= a.row_count) return;
    const uint32_t r = token - a.first_row;
    const uint8_t* s[F::kStreams];
#pragma unroll
    for (int q = 0; q < F::kStreams; ++q)
        s[q] = static_cast<const uint8_t*>(a.piece) + RowStreams<F>::base(q, a.blocks) + static_cast<uint64_t>(r) * RowStreams<F>::row_bytes(q, a.width / 32u);
    F f;
    f.load(s, g);
    float w[32];
    put_all<F>(f, a.scale, w, std::make_integer_sequence<int, 32>{});
    float4* out = reinterpret_cast<float4*>(a.hidden + static_cast<size_t>(row) * a.width + g * 32u);
#pragma unroll
    for (int v = 0; v < 8; ++v) out[v] = make_float4(w[4 * v], w[4 * v + 1], w[4 * v + 2], w[4 * v + 3]);
}

template <typename F>
cudaError_t launch(const GatherArgs& a, cudaStream_t stream, bool pdl) {
    const uint32_t n = a.tokens * (a.width / 32u);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((n + 127u) / 128u);
    cfg.blockDim = dim3(128);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gather_kernel<F>, a);
}

}  // namespace

cudaError_t gather_run(const GatherArgs& a, cudaStream_t stream, bool pdl) {
    switch (a.format) {
        case kQ4_0: return launch<Q4_0>(a, stream, pdl);
        case kQ8_0: return launch<Q8_0>(a, stream, pdl);
        case kQ6_K: return launch<Q6_K>(a, stream, pdl);
        case kQ4_1: return launch<Q4_1>(a, stream, pdl);
        case kBF16: return launch<BF16>(a, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace cb
