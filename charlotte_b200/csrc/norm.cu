// RMSNorm with the residual add before it (plainsight-systems/charlotte,
// src/core/kernels/norm/norm.wgsl:80-198; launcher norm.h:189-220).
//
// One CTA of 256 threads a row, as the reference's workgroup: thread i holds
// the row's vec4s i, i+256, ... (up to 4), sums its squares with `+ dot`,
// and the 256 partial sums meet in the reference's tree — halving at each
// level, partial[i] += partial[i + stride]. Levels of stride >= 32 go
// through shared memory; below that a shuffle-down by `stride` pairs exactly
// the same elements, so the total's bits are the tree's. Then
// r = 1/sqrt(total/n + eps) and normed = (x·r)·g.
//
// With `add`, y (the block's output) is added first — post-normed with its
// own gain when the layer has a post-norm (Gemma 3) — then x times `scale`
// when given (Gemma 4's layer output scale), and the new hidden row written
// back; `add_only` stops there. `last_token` normalizes only the step's last
// row (the final norm); `rows_per_token` rows a token are each their own
// row (the per-layer inputs); without a gain, normed = x·r (unit_gain).
// Rows ≤ 4096 wide, a multiple of 4.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"
#include "numerics.cuh"
#include "tma.cuh"

namespace cb {

namespace {

constexpr int kNormThreads = 256;
constexpr int kMaxVec4 = 4;

// The reference's reduce (norm.wgsl:67-78): returns the tree's total to
// every thread. `scratch` holds 256 floats.
__device__ __forceinline__ float tree_sum(float v, float* scratch) {
    const int i = threadIdx.x;
    scratch[i] = v;
    __syncthreads();
#pragma unroll
    for (int stride = kNormThreads / 2; stride >= 32; stride >>= 1) {
        if (i < stride) scratch[i] = scratch[i] + scratch[i + stride];
        __syncthreads();
    }
    if (i < 32) {
        float w = scratch[i];
#pragma unroll
        for (int stride = 16; stride > 0; stride >>= 1) w = w + __shfl_down_sync(0xFFFFFFFFu, w, stride);
        if (i == 0) scratch[0] = w;
    }
    __syncthreads();
    const float total = scratch[0];
    __syncthreads();   // every thread has read it before the next reduction writes
    return total;
}

__global__ void __launch_bounds__(kNormThreads) norm_kernel(NormArgs a) {
    __shared__ float scratch[kNormThreads];
    grid_dependency_wait();
    const uint32_t row = a.last_token ? a.tokens - 1u : blockIdx.x;
    const uint32_t vec4s = a.width / 4u;
    const size_t base = static_cast<size_t>(row) * vec4s;
    const float n = static_cast<float>(a.width);
    float4* hidden = reinterpret_cast<float4*>(a.hidden) + base;
    const float4* gain = reinterpret_cast<const float4*>(a.gain);
    float4 x[kMaxVec4];
#pragma unroll
    for (int k = 0; k < kMaxVec4; ++k) {
        const uint32_t i = threadIdx.x + k * kNormThreads;
        x[k] = i < vec4s ? hidden[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (a.add) {
        const float4* out = reinterpret_cast<const float4*>(a.output) + base;
        float4 y[kMaxVec4];
#pragma unroll
        for (int k = 0; k < kMaxVec4; ++k) {
            const uint32_t i = threadIdx.x + k * kNormThreads;
            y[k] = i < vec4s ? out[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        if (a.post_gain) {
            float squares = 0.0f;
#pragma unroll
            for (int k = 0; k < kMaxVec4; ++k)
                if (threadIdx.x + k * kNormThreads < vec4s) squares = squares + dot4(y[k], y[k]);
            const float r = 1.0f / sqrtf(tree_sum(squares, scratch) / n + a.epsilon);
            const float4* pg = reinterpret_cast<const float4*>(a.post_gain);
#pragma unroll
            for (int k = 0; k < kMaxVec4; ++k) {
                const uint32_t i = threadIdx.x + k * kNormThreads;
                if (i < vec4s) {
                    const float4 g = pg[i];
                    y[k] = make_float4(((y[k].x * r) * g.x) * 1.0f, ((y[k].y * r) * g.y) * 1.0f,
                                       ((y[k].z * r) * g.z) * 1.0f, ((y[k].w * r) * g.w) * 1.0f);
                }
            }
        }
        const float sc = a.scale ? *a.scale : 1.0f;
#pragma unroll
        for (int k = 0; k < kMaxVec4; ++k) {
            const uint32_t i = threadIdx.x + k * kNormThreads;
            if (i < vec4s) {
                x[k] = make_float4(x[k].x + y[k].x, x[k].y + y[k].y, x[k].z + y[k].z, x[k].w + y[k].w);
                if (a.scale) x[k] = make_float4(x[k].x * sc, x[k].y * sc, x[k].z * sc, x[k].w * sc);
                hidden[i] = x[k];
            }
        }
        if (a.add_only) {
            grid_dependents_launch();
            return;
        }
    }
    float squares = 0.0f;
#pragma unroll
    for (int k = 0; k < kMaxVec4; ++k)
        if (threadIdx.x + k * kNormThreads < vec4s) squares = squares + dot4(x[k], x[k]);
    const float r = 1.0f / sqrtf(tree_sum(squares, scratch) / n + a.epsilon);
    grid_dependents_launch();
    float4* normed = reinterpret_cast<float4*>(a.normed) + base;
#pragma unroll
    for (int k = 0; k < kMaxVec4; ++k) {
        const uint32_t i = threadIdx.x + k * kNormThreads;
        if (i < vec4s) {
            float4 v;
            if (gain) {
                const float4 g = gain[i];
                v = make_float4((x[k].x * r) * g.x, (x[k].y * r) * g.y, (x[k].z * r) * g.z, (x[k].w * r) * g.w);
            } else {
                v = make_float4(x[k].x * r, x[k].y * r, x[k].z * r, x[k].w * r);
            }
            normed[i] = v;
            if (a.normed16) {
                __half2* h = reinterpret_cast<__half2*>(a.normed16) + 2u * (base + i);
                h[0] = __floats2half2_rn(v.x, v.y);
                h[1] = __floats2half2_rn(v.z, v.w);
            }
        }
    }
}

}  // namespace

cudaError_t norm_run(const NormArgs& a, cudaStream_t stream, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.last_token ? 1u : a.tokens * (a.rows_per_token > 1u ? a.rows_per_token : 1u));
    cfg.blockDim = dim3(kNormThreads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, norm_kernel, a);
}

}  // namespace cb
