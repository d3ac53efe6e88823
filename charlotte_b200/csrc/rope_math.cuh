// The per-token and per-head arithmetic of the QK-norm, RoPE and KV append
// (plainsight-systems/charlotte, src/core/kernels/rope/rope.wgsl +
// rope_cache.wgsl:11-89), shared by the rope launch (rope.cu) and the decode
// attention that folds the step's rope into its prologue (attention.cu), so
// both give the same bits.
#pragma once

#include <cstdint>

#include "numerics.cuh"

namespace cb {

// The token's angle table for position p: t = p·turn_k (then t/factor_k
// with llama3 factors), angle = 2π·(t − round_even(t)), and its sine and
// cosine (Cody–Waite/Taylor, numerics.cuh); entries k = first, first+step, ...
// Entry k from its turn and factor (factor used only when `scaled`).
__device__ __forceinline__ void rope_angle(uint32_t p, float turn, float factor, bool scaled, float* cosine,
                                           float* sine) {
    float t = static_cast<float>(p) * turn;
    if (scaled) t = t / factor;
    const float angle = 6.283185307179586f * (t - rintf(t));
    sincos_turn(angle, sine, cosine);
}

__device__ __forceinline__ void rope_angles(uint32_t p, const float* turns, const float* factors, uint32_t d,
                                            float* cosines, float* sines, uint32_t first, uint32_t step) {
    for (uint32_t k = first; k < d / 2u; k += step)
        rope_angle(p, turns[k], factors ? factors[k] : 1.0f, factors != nullptr, &cosines[k], &sines[k]);
}

// One head held by `lanes` = d/8 threads, lane i holding vec4s i and
// i + lanes, as the reference's invocations do. With `norm`, the QK-norm's
// sum dot(a,a) + dot(b,b) over the head's lanes in the reference's halving
// tree (reduce_head, rope.wgsl:62-73: a shuffle-down by `stride` within the
// head's lanes pairs the same elements), r = 1/sqrt(total/d + epsilon), and
// with `gain` (x·r)·g; with `turn`, the pairs turned by their angle — NEOX
// halves or adjacent pairs. Every lane of the warp calls it (the shuffles
// span the warp); value heads pass no gain and no turn.
// A head's 1/sqrt(mean square + epsilon) from its lanes' vec4 pairs, the
// sum in reduce_head's tree; every lane of the warp takes part.
__device__ __forceinline__ float head_norm_factor(float4 x0, float4 x1, uint32_t lanes, uint32_t d, float epsilon) {
    float v = dot4(x0, x0) + dot4(x1, x1);
    for (uint32_t stride = lanes / 2u; stride > 0; stride >>= 1) v = v + __shfl_down_sync(0xFFFFFFFFu, v, stride, lanes);
    const float total = __shfl_sync(0xFFFFFFFFu, v, 0, lanes);
    return 1.0f / sqrtf(total / static_cast<float>(d) + epsilon);
}

__device__ __forceinline__ void rope_head(float4& x0, float4& x1, uint32_t lane, uint32_t lanes, uint32_t d,
                                          bool norm, float epsilon, const float* gain, bool turn, bool halves,
                                          const float* cosines, const float* sines) {
    float r = 1.0f;
    if (norm) r = head_norm_factor(x0, x1, lanes, d, epsilon);
    if (!turn) return;
    if (gain) {
        const float4 g0 = reinterpret_cast<const float4*>(gain)[lane];
        const float4 g1 = reinterpret_cast<const float4*>(gain)[lane + lanes];
        x0 = make_float4((x0.x * r) * g0.x, (x0.y * r) * g0.y, (x0.z * r) * g0.z, (x0.w * r) * g0.w);
        x1 = make_float4((x1.x * r) * g1.x, (x1.y * r) * g1.y, (x1.z * r) * g1.z, (x1.w * r) * g1.w);
    }
    if (halves) {
        // pairs k = 4·lane + c: (x0.c, x1.c) turned by angle k
        float* e0 = &x0.x;
        float* e1 = &x1.x;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint32_t k = 4u * lane + c;
            const float u = e0[c], w = e1[c];
            e0[c] = fmaf(u, cosines[k], -(w * sines[k]));
            e1[c] = fmaf(u, sines[k], w * cosines[k]);
        }
    } else {
        // adjacent pairs: x0 holds pairs 2·lane, 2·lane+1; x1 pairs d/4 + 2·lane, +1
        float* e[2] = {&x0.x, &x1.x};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const uint32_t k = (h ? d / 4u : 0u) + 2u * lane + c;
                const float u = e[h][2 * c], w = e[h][2 * c + 1];
                e[h][2 * c] = fmaf(u, cosines[k], (-w) * sines[k]);
                e[h][2 * c + 1] = fmaf(w, cosines[k], u * sines[k]);
            }
        }
    }
}

// Four floats packed f16 (saturated to ±65,504, round to nearest even).
__device__ __forceinline__ void store_f16x4(uint16_t* dst, float4 v) {
    const uint32_t lo = static_cast<uint32_t>(f32_to_f16_sat(v.x)) | (static_cast<uint32_t>(f32_to_f16_sat(v.y)) << 16);
    const uint32_t hi = static_cast<uint32_t>(f32_to_f16_sat(v.z)) | (static_cast<uint32_t>(f32_to_f16_sat(v.w)) << 16);
    *reinterpret_cast<uint2*>(dst) = make_uint2(lo, hi);
}

}  // namespace cb
