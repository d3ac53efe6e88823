// An encoder's own kernels (plainsight-systems/charlotte, src/core/graph/
// encoder.h): block attention (block_attention.wgsl scores_of :95 + weigh
// :205, launcher block_attention.h:333) and pooling (pool.wgsl mean :49 and
// unit :63, launcher pool.h:107-121).
//
// Block attention, every row of a step attending to every row within the
// layer's half window either side, computed as the reference orders it:
//   s_ij = (dot4(q_0, k_0) + dot4(q_1, k_1) + … along d, a chain from 0) ×
//          scale·log2e;
//   m_i  = the largest live score of the row (max is exact: any order);
//   p_ij = exp2(s_ij − m_i) (attention's exp2);
//   O_i  = fma(p_ij, v_j, O_i) and l_i = l_i + p_ij over the live keys in
//          order; out = O_i / l_i.
// The reference writes every score to a buffer between its two launches;
// here one launch keeps a CTA's rows' scores in shared memory. A CTA a (kv
// head, block of 16/G rows × G heads = 16 query vectors): the vectors and a
// 32-key chunk of keys staged (key rows padded by one float4, so the lanes'
// keys fall on distinct banks), a thread a key × 2 vectors for the scores;
// a warp a vector for the maxima; a thread a (vector, 4 dimensions) for the
// weighted sums, values read straight from L2, coalesced along d. Keys that
// are not live add exact zeros in the reference (fma(0, v, O) = O; O is
// never −0), so only each row's live range is walked.
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"
#include "numerics.cuh"
#include "tma.cuh"

namespace cb {

namespace {

constexpr uint32_t kBlockVectors = 16;   // query vectors a CTA
constexpr uint32_t kBlockKeys = 32;      // keys a staged chunk
constexpr uint32_t kBlockThreads = 256;

size_t block_smem(uint32_t d, uint32_t tokens) {
    return (static_cast<size_t>(kBlockVectors) * d + static_cast<size_t>(kBlockKeys) * (d + 4u) +
            static_cast<size_t>(kBlockVectors) * tokens) *
           sizeof(float);
}

__global__ void __launch_bounds__(kBlockThreads) block_attention_kernel(const cb_block_attention a) {
    extern __shared__ __align__(16) float bsm[];
    const uint32_t d = a.head_dim, n = a.tokens, quads = d / 4u;
    const uint32_t G = a.query_heads / a.kv_heads;
    const uint32_t kv = blockIdx.x, rows = kBlockVectors / G;
    const uint32_t row0 = blockIdx.y * rows;
    const uint32_t t = threadIdx.x, lane = t & 31u, warp = t >> 5;
    float* qs = bsm;                                    // [16][d]
    float* ks = qs + kBlockVectors * d;                 // [32][d + 4]
    float* ss = ks + kBlockKeys * (d + 4u);             // [16][n]: scores, then weights
    const uint32_t kstride = d + 4u;
    grid_dependency_wait();

    // Vector v: row row0 + v / G, query head kv·G + v % G.
    auto row_of = [&](uint32_t v) { return row0 + v / G; };
    auto head_of = [&](uint32_t v) { return kv * G + v % G; };
    auto lo_of = [&](uint32_t i) { return i > a.half_window ? i - a.half_window : 0u; };
    auto hi_of = [&](uint32_t i) { return (n - 1u - i) > a.half_window ? i + a.half_window : n - 1u; };

    for (uint32_t e = t; e < kBlockVectors * quads; e += kBlockThreads) {
        const uint32_t v = e / quads, c = e % quads;
        const uint32_t i = row_of(v);
        float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i < n) q = reinterpret_cast<const float4*>(a.query + (static_cast<size_t>(i) * a.query_heads + head_of(v)) * d)[c];
        reinterpret_cast<float4*>(qs + v * d)[c] = q;
    }
    // The keys any of the CTA's rows sees.
    const uint32_t last_row = min(row0 + rows, n) - 1u;
    const uint32_t k_lo = lo_of(row0), k_hi = hi_of(last_row);
    const uint32_t v0 = warp, v1 = warp + 8u;   // this thread's two vectors
    for (uint32_t j0 = k_lo / kBlockKeys * kBlockKeys; j0 <= k_hi; j0 += kBlockKeys) {
        __syncthreads();   // the last chunk's keys are read
        for (uint32_t e = t; e < kBlockKeys * quads; e += kBlockThreads) {
            const uint32_t b = e / quads, c = e % quads, j = j0 + b;
            float4 k = make_float4(0.f, 0.f, 0.f, 0.f);
            if (j < n) k = reinterpret_cast<const float4*>(a.key + (static_cast<size_t>(j) * a.kv_heads + kv) * d)[c];
            reinterpret_cast<float4*>(ks + b * kstride)[c] = k;
        }
        __syncthreads();
        const uint32_t j = j0 + lane;
        const float4* kr = reinterpret_cast<const float4*>(ks + lane * kstride);
        const float4* q0 = reinterpret_cast<const float4*>(qs + v0 * d);
        const float4* q1 = reinterpret_cast<const float4*>(qs + v1 * d);
        float acc0 = 0.0f, acc1 = 0.0f;
        for (uint32_t c = 0; c < quads; ++c) {
            const float4 k = kr[c];
            acc0 = acc0 + dot4(q0[c], k);
            acc1 = acc1 + dot4(q1[c], k);
        }
        if (j < n) {
            ss[v0 * n + j] = acc0 * a.scale_log2e;
            ss[v1 * n + j] = acc1 * a.scale_log2e;
        }
    }
    __syncthreads();
    grid_dependents_launch();

    // Each vector's largest live score, then its weights in place.
    for (uint32_t v = warp; v < kBlockVectors; v += kBlockThreads / 32u) {
        const uint32_t i = row_of(v);
        if (i >= n) continue;
        const uint32_t lo = lo_of(i), hi = hi_of(i);
        float m = -__int_as_float(0x7f800000);
        for (uint32_t j = lo + lane; j <= hi; j += 32u) m = fmaxf(m, ss[v * n + j]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, off));
        for (uint32_t j = lo + lane; j <= hi; j += 32u) ss[v * n + j] = exp2_np(ss[v * n + j] - m);
    }
    __syncthreads();

    // O = fma(p, v, O) and l = l + p over the live keys in order; out = O / l.
    for (uint32_t e = t; e < kBlockVectors * quads; e += kBlockThreads) {
        const uint32_t v = e / quads, c = e % quads;
        const uint32_t i = row_of(v);
        if (i >= n) continue;
        const uint32_t lo = lo_of(i), hi = hi_of(i);
        const float* p = ss + v * n;
        const float4* val = reinterpret_cast<const float4*>(a.value + static_cast<size_t>(kv) * d) + c;
        const size_t step = static_cast<size_t>(a.kv_heads) * quads;
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        float l = 0.0f;
        for (uint32_t j = lo; j <= hi; ++j) {
            const float w = p[j];
            const float4 x = __ldg(val + j * step);
            o = make_float4(fmaf(w, x.x, o.x), fmaf(w, x.y, o.y), fmaf(w, x.z, o.z), fmaf(w, x.w, o.w));
            l = l + w;
        }
        reinterpret_cast<float4*>(a.out + (static_cast<size_t>(i) * a.query_heads + head_of(v)) * d)[c] =
            make_float4(o.x / l, o.y / l, o.z / l, o.w / l);
    }
}

// pool.wgsl mean: column c's chain of adds down the rows, times 1/n, at
// row n − 1 of the output.
__global__ void __launch_bounds__(256) pool_mean_kernel(const cb_pool p) {
    grid_dependency_wait();
    const uint32_t vec4s = p.width / 4u, n = p.tokens;
    const float inverse = 1.0f / static_cast<float>(n);
    const float4* in = reinterpret_cast<const float4*>(p.input);
    float4* out = reinterpret_cast<float4*>(p.output) + static_cast<size_t>(n - 1u) * vec4s;
    for (uint32_t c = blockIdx.x * blockDim.x + threadIdx.x; c < vec4s; c += gridDim.x * blockDim.x) {
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
        for (uint32_t r = 0; r < n; ++r) {
            const float4 x = in[static_cast<size_t>(r) * vec4s + c];
            s = make_float4(s.x + x.x, s.y + x.y, s.z + x.z, s.w + x.w);
        }
        out[c] = make_float4(s.x * inverse, s.y * inverse, s.z * inverse, s.w * inverse);
    }
    grid_dependents_launch();
}

// pool.wgsl unit: the squares of thread i's vec4s i, i + 256, … in order,
// the 256 partial sums in the norm's halving tree, r = 1/sqrt(total) (0 for
// a zero row), each element × r.
__global__ void __launch_bounds__(256) pool_unit_kernel(const cb_pool p) {
    __shared__ float partial[256];
    grid_dependency_wait();
    const uint32_t vec4s = p.width / 4u, i = threadIdx.x;
    const float4* in = reinterpret_cast<const float4*>(p.input);
    float4 x[4];
    float squares = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t c = i + 256u * k;
        x[k] = c < vec4s ? in[c] : make_float4(0.f, 0.f, 0.f, 0.f);
        if (c < vec4s) squares = squares + dot4(x[k], x[k]);
    }
    partial[i] = squares;
    __syncthreads();
    for (uint32_t stride = 128; stride > 0; stride >>= 1) {
        if (i < stride) partial[i] = partial[i] + partial[i + stride];
        __syncthreads();
    }
    const float total = partial[0];
    const float r = total > 0.0f ? 1.0f / sqrtf(total) : 0.0f;
    grid_dependents_launch();
    float4* out = reinterpret_cast<float4*>(p.output);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t c = i + 256u * k;
        if (c < vec4s) out[c] = make_float4(x[k].x * r, x[k].y * r, x[k].z * r, x[k].w * r);
    }
}

cudaLaunchConfig_t config(dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                          cudaLaunchAttribute* attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cfg;
}

}  // namespace

bool block_attention_fits(const cb_block_attention& a) {
    return block_smem(a.head_dim, a.tokens) <= 200u * 1024u;
}

cudaError_t block_attention_run(const cb_block_attention& a, cudaStream_t stream, bool pdl) {
    const size_t smem = block_smem(a.head_dim, a.tokens);
    static size_t configured = 0;
    if (smem > configured) {
        const cudaError_t e = cudaFuncSetAttribute(block_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        configured = smem;
    }
    const uint32_t rows = kBlockVectors / (a.query_heads / a.kv_heads);
    cudaLaunchAttribute attr[1];
    const cudaLaunchConfig_t cfg =
        config(dim3(a.kv_heads, (a.tokens + rows - 1u) / rows), dim3(kBlockThreads), smem, stream, pdl, attr);
    return cudaLaunchKernelEx(&cfg, block_attention_kernel, a);
}

cudaError_t pool_run(const cb_pool& p, cudaStream_t stream, bool pdl) {
    cudaLaunchAttribute attr[1];
    if (p.kind == CB_POOL_MEAN) {
        const uint32_t vec4s = p.width / 4u;
        const cudaLaunchConfig_t cfg = config(dim3((vec4s + 255u) / 256u), dim3(256), 0, stream, pdl, attr);
        return cudaLaunchKernelEx(&cfg, pool_mean_kernel, p);
    }
    const cudaLaunchConfig_t cfg = config(dim3(1), dim3(256), 0, stream, pdl, attr);
    return cudaLaunchKernelEx(&cfg, pool_unit_kernel, p);
}

}  // namespace cb
