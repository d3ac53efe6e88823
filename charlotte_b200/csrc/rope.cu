// QK-norm, RoPE and the KV append (plainsight-systems/charlotte,
// src/core/kernels/rope/rope.wgsl + rope_cache.wgsl:11-89; launcher
// rope.h:282-300, rope.cpp:76-87, 107-130).
//
// One CTA a token row: (Hq + 2·Hkv) heads × d/8 lanes, lane i of a head
// holding its vec4s i and i + d/8, as the reference's invocations do. The
// token's angles are computed once into shared memory: t = p·turn_k (then
// t/factor_k with llama3 factors), angle = 2π·(t − round_even(t)), and its
// sine and cosine by the Cody–Waite/Taylor method of numerics.cuh. A query
// or key head with QK-norm sums dot(a,a) + dot(b,b) over its lanes in the
// reference's halving tree (reduce_head, rope.wgsl:62-73; a shuffle-down by
// `stride` within the head's lanes pairs the same elements), then
// (x·r)·g. Query and key pairs turn by their angle — NEOX halves or
// adjacent pairs — queries written back f32, keys and values packed f16
// (saturated, round-to-nearest-even) into slot p mod slots. The encode form
// (rope_encode.wgsl, an encoder's) writes keys back f32 in place instead,
// and with value_norm scales each value head by its 1/sqrt(mean square +
// epsilon); no cache.
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"
#include "numerics.cuh"
#include "rope_math.cuh"
#include "tma.cuh"

namespace cb {

namespace {

__global__ void rope_kernel(RopeArgs a) {
    extern __shared__ float angles[];   // cos then sin, d/2 each
    grid_dependency_wait();
    const uint32_t d = a.head_dim;
    const uint32_t lanes = d / 8u;
    const uint32_t row = blockIdx.x;
    // Rows are consecutive positions of one sequence, or (batched decode)
    // one token each of `tokens` sequences at the step's position.
    const uint32_t p = (a.position ? *a.position : a.position0) + (a.rows_are_sequences ? 0u : row);
    float* cosines = angles;
    float* sines = angles + d / 2u;
    rope_angles(p, a.turns, a.factors, d, cosines, sines, threadIdx.x, blockDim.x);
    __syncthreads();
    grid_dependents_launch();

    const uint32_t head = threadIdx.x / lanes;
    const uint32_t lane = threadIdx.x % lanes;
    const uint32_t hq = a.query_heads, hkv = a.kv_heads;
    if (head >= hq + 2u * hkv) return;
    const bool is_query = head < hq;
    const bool is_value = head >= hq + hkv;
    const uint32_t kvh = is_value ? head - hq - hkv : head - hq;
    const float4* src;
    if (is_query) src = reinterpret_cast<const float4*>(a.query + (static_cast<size_t>(row) * hq + head) * d);
    else if (is_value) src = reinterpret_cast<const float4*>(a.value + (static_cast<size_t>(row) * hkv + kvh) * d);
    else src = reinterpret_cast<const float4*>(a.key + (static_cast<size_t>(row) * hkv + kvh) * d);
    float4 x0 = src[lane];
    float4 x1 = src[lane + lanes];

    if (a.encode) {
        // rope_encode.wgsl: keys turned like queries and written back in
        // place; value heads normalized without a gain (value_norm). The
        // reduce runs on every lane where either needs it (uniform).
        const bool qk = a.query_gain != nullptr, vn = a.value_norm != 0;
        float r = 1.0f;
        if ((qk || vn) && lanes <= 32u) {
            r = head_norm_factor(x0, x1, lanes, d, a.epsilon);
        } else if (qk || vn) {
            // Heads of 512: 64 lanes over two warps. reduce_head's first
            // level (stride 32) through shared memory, the rest within the
            // head's first warp, the total back through shared memory.
            float* red = angles + d;                 // a float a thread
            float* total = red + blockDim.x;         // a float a head
            float v = dot4(x0, x0) + dot4(x1, x1);
            red[threadIdx.x] = v;
            __syncthreads();
            if (lane < 32u) {
                v = v + red[threadIdx.x + 32u];
                for (uint32_t stride = 16u; stride > 0; stride >>= 1) v = v + __shfl_down_sync(0xFFFFFFFFu, v, stride);
                if (lane == 0) total[head] = v;
            }
            __syncthreads();
            r = 1.0f / sqrtf(total[head] / static_cast<float>(d) + a.epsilon);
        }
        if (!is_value) {
            if (qk) {   // (x·r)·g, then the turn: the decoder form's steps
                const float4* g = reinterpret_cast<const float4*>(is_query ? a.query_gain : a.key_gain);
                const float4 g0 = g[lane], g1 = g[lane + lanes];
                x0 = make_float4((x0.x * r) * g0.x, (x0.y * r) * g0.y, (x0.z * r) * g0.z, (x0.w * r) * g0.w);
                x1 = make_float4((x1.x * r) * g1.x, (x1.y * r) * g1.y, (x1.z * r) * g1.z, (x1.w * r) * g1.w);
            }
            rope_head(x0, x1, lane, lanes, d, false, a.epsilon, nullptr, true, a.halves != 0, cosines, sines);
        } else if (vn) {
            x0 = make_float4(x0.x * r, x0.y * r, x0.z * r, x0.w * r);
            x1 = make_float4(x1.x * r, x1.y * r, x1.z * r, x1.w * r);
        }
        float* base = is_query ? a.query + (static_cast<size_t>(row) * hq + head) * d
                               : (is_value ? a.value : a.key) + (static_cast<size_t>(row) * hkv + kvh) * d;
        reinterpret_cast<float4*>(base)[lane] = x0;
        reinterpret_cast<float4*>(base)[lane + lanes] = x1;
        return;
    }
    // QK-norm (uniform over the CTA: both gains or neither). Every lane takes
    // part in the shuffles — a warp may hold a key head and a value head —
    // and value heads discard the result.
    rope_head(x0, x1, lane, lanes, d, a.query_gain != nullptr, a.epsilon, is_query ? a.query_gain : a.key_gain,
              !is_value, a.halves != 0, cosines, sines);
    if (is_query) {
        float4* dst = reinterpret_cast<float4*>(a.query + (static_cast<size_t>(row) * hq + head) * d);
        dst[lane] = x0;
        dst[lane + lanes] = x1;
    } else {
        uint16_t* cache = (is_value ? a.value_cache : a.key_cache) +
                          (a.rows_are_sequences ? static_cast<size_t>(row) * a.sequence_stride : 0u);
        uint16_t* dst = cache + (static_cast<size_t>(p % a.slots) * hkv + kvh) * d;
        store_f16x4(dst + 4u * lane, x0);
        store_f16x4(dst + 4u * (lane + lanes), x1);
    }
}

}  // namespace

cudaError_t rope_run(const RopeArgs& a, cudaStream_t stream, bool pdl) {
    const uint32_t threads = (a.query_heads + 2u * a.kv_heads) * (a.head_dim / 8u);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.tokens);
    cfg.blockDim = dim3((threads + 31u) / 32u * 32u);
    // the angles; heads of 512 (encode form) also a reduce float a thread and a total a head
    cfg.dynamicSmemBytes = (a.head_dim + (a.head_dim > 256u ? threads + a.query_heads + 2u * a.kv_heads : 0u)) *
                           sizeof(float);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, rope_kernel, a);
}

}  // namespace cb
