// Attention for steps of many query rows (prefill), over the f16 KV cache:
// the same arithmetic as attention.cu (plainsight-systems/charlotte,
// src/core/kernels/attention/attention.wgsl main :138-360, fold :101-127),
// query by query, bit for bit — chunks of 64 keys fixed by position, tiles of
// B = 2048/d keys within a chunk, online softmax in log2 units, chunks folded
// in chunk order — laid out for many queries instead of many keys.
//
// B200 mapping: a CTA per (kv head, tile of Q queries: Q/G rows × the G query
// heads of the kv head), Q = 64 (32 for d = 256). The CTA walks the tile's
// chunks in order; each chunk's keys and values are staged in shared memory
// once for all Q queries, and each query's running state (m, l, O) stays in
// shared memory across chunks, so there are no partials and no second pass:
// a chunk's P·V is folded into O as soon as it is formed, which is the
// reference's chunk order. Per chunk:
//   1. scores, a thread 4 queries × 4 keys, s = Σ_w dot(q_w, k_w) in order;
//   2. each (query, tile): the tile's top over its live scores;
//   3. each query, tiles in order: top, alpha, the chunk's running max;
//   4. each (query, tile): the weights 2^(s − top) and their sum in key order;
//   5. each query: the chunk's l, then the fold factors against the run;
//   6. P·V, a thread 4 queries × 8 dimensions, tiles in order, each tile's
//      alpha then fma over its keys in order, then the fold into O.
// Keys not live for a query, and weights that are exactly zero, are skipped,
// as the oracle skips them, so zeros keep their signs.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"
#include "numerics.cuh"
#include "tma.cuh"

namespace cb {

namespace {

constexpr uint32_t kChunk = 64;
constexpr uint32_t kThreads = 256;

template <uint32_t D>
struct Prefill {
    static constexpr uint32_t Q = D <= 128 ? 64u : 32u;   // queries a CTA
    static constexpr uint32_t B = 2048u / D;               // keys a tile
    static constexpr uint32_t T = kChunk / B;              // tiles a chunk
    static constexpr uint32_t QS = D + 4;                  // floats a staged query row
    static constexpr uint32_t KS = D + 4;                  // halves a staged key row (8-byte rows, no bank conflict)
    static constexpr uint32_t VS = D;                      // halves a staged value row
    static constexpr uint32_t PS = Q + 4;                  // floats a row of P (one key, every query)
    // shared memory, in floats
    static constexpr uint32_t kQ = 0;
    static constexpr uint32_t kK = kQ + Q * QS;
    static constexpr uint32_t kV = kK + kChunk * KS / 2;
    static constexpr uint32_t kP = kV + kChunk * VS / 2;
    static constexpr uint32_t kO = kP + kChunk * PS;
    static constexpr uint32_t kTile = kO + Q * D;          // [5][Q][T]: tmax, seen, top, alpha, tsum
    static constexpr uint32_t kQuery = kTile + 5 * Q * T;  // [8][Q]: run_m, run_l, run_live, fa, fb, fold, chunk_m, p
    static constexpr uint32_t kFloats = kQuery + 8 * Q;
    static constexpr size_t kSmem = kFloats * 4ull;
    static_assert(kSmem <= 200u * 1024u, "");
};

__device__ __forceinline__ uint32_t earliest_of(uint32_t p, uint32_t window) {
    return p + 1u > window ? p + 1u - window : 0u;
}

template <uint32_t D>
__global__ void __launch_bounds__(kThreads) attention_prefill_kernel(const AttentionArgs a) {
    using P = Prefill<D>;
    constexpr uint32_t Q = P::Q, B = P::B, T = P::T;
    extern __shared__ __align__(16) float sm[];
    float* qs = sm + P::kQ;
    uint16_t* ks = reinterpret_cast<uint16_t*>(sm + P::kK);
    uint16_t* vs = reinterpret_cast<uint16_t*>(sm + P::kV);
    float* ps = sm + P::kP;
    float* orun = sm + P::kO;
    float* t_max = sm + P::kTile;
    float* t_seen = t_max + Q * T;
    float* t_top = t_seen + Q * T;
    float* t_alpha = t_top + Q * T;
    float* t_sum = t_alpha + Q * T;
    float* run_m = sm + P::kQuery;
    float* run_l = run_m + Q;
    float* run_live = run_l + Q;
    float* f_a = run_live + Q;
    float* f_b = f_a + Q;
    float* f_fold = f_b + Q;
    float* c_m = f_fold + Q;
    uint32_t* q_pos = reinterpret_cast<uint32_t*>(c_m + Q);

    const uint32_t tid = threadIdx.x;
    const uint32_t G = a.query_heads / a.kv_heads;
    const uint32_t R = Q / G;                          // rows a tile
    const uint32_t kvh = blockIdx.x;
    const uint32_t row0 = blockIdx.y * R;
    const uint32_t rows = min(R, a.tokens - row0);
    const uint32_t nq = rows * G;                      // live queries of the tile

    grid_dependency_wait();
    const uint32_t pos0 = a.position ? *a.position : a.position0;
    const uint32_t p_first = pos0 + row0, p_last = pos0 + row0 + rows - 1u;

    // Queries m = r·G + g (row r, head kvh·G + g), scaled into log2 units;
    // the running state empty.
    for (uint32_t i = tid; i < Q * (D / 4u); i += kThreads) {
        const uint32_t m = i / (D / 4u), w = i % (D / 4u);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (m < nq) {
            const uint32_t r = m / G, h = kvh * G + m % G;
            v = __ldcg(reinterpret_cast<const float4*>(a.query + (static_cast<size_t>(row0 + r) * a.query_heads + h) * D) + w);
            v.x = v.x * a.scale_log2e; v.y = v.y * a.scale_log2e;
            v.z = v.z * a.scale_log2e; v.w = v.w * a.scale_log2e;
        }
        *reinterpret_cast<float4*>(qs + m * P::QS + 4u * w) = v;
    }
    for (uint32_t i = tid; i < Q * D; i += kThreads) orun[i] = 0.0f;
    if (tid < Q) {
        run_m[tid] = 0.0f;
        run_l[tid] = 0.0f;
        run_live[tid] = 0.0f;
        q_pos[tid] = pos0 + row0 + min(tid / G, rows - 1u);
    }

    const uint32_t c_lo = earliest_of(p_first, a.window) / kChunk, c_hi = p_last / kChunk;
    for (uint32_t c = c_lo; c <= c_hi; ++c) {
        const uint32_t key0 = c * kChunk;
        const uint32_t j_lo = max(key0, earliest_of(p_first, a.window));
        const uint32_t j_hi = min(key0 + kChunk, p_last + 1u);   // staged keys [j_lo, j_hi)
        __syncthreads();   // the last chunk's reads of ks, vs, ps are done; the set-up above is visible
        // Stage keys (8-byte words: rows of D+4 halves) and values (16-byte words).
        for (uint32_t i = tid; i < (j_hi - j_lo) * (D / 4u); i += kThreads) {
            const uint32_t b = j_lo - key0 + i / (D / 4u), w = i % (D / 4u);
            const size_t at = (static_cast<size_t>((key0 + b) % a.slots) * a.kv_heads + kvh) * D;
            *reinterpret_cast<uint2*>(ks + b * P::KS + 4u * w) = __ldcg(reinterpret_cast<const uint2*>(a.key_cache + at) + w);
        }
        for (uint32_t i = tid; i < (j_hi - j_lo) * (D / 8u); i += kThreads) {
            const uint32_t b = j_lo - key0 + i / (D / 8u), w = i % (D / 8u);
            const size_t at = (static_cast<size_t>((key0 + b) % a.slots) * a.kv_heads + kvh) * D;
            *reinterpret_cast<uint4*>(vs + b * P::VS + 8u * w) = __ldcg(reinterpret_cast<const uint4*>(a.value_cache + at) + w);
        }
        __syncthreads();

        // 1. Scores: queries 4mq..4mq+3, keys kq + 16i.
        for (uint32_t task = tid; task < (Q / 4u) * 16u; task += kThreads) {
            const uint32_t kq = task % 16u, mq = task / 16u;
            float s[4][4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int k = 0; k < 4; ++k) s[i][k] = 0.0f;
#pragma unroll 4
            for (uint32_t w = 0; w < D / 4u; ++w) {
                float4 kf[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const uint2 kw = *reinterpret_cast<const uint2*>(ks + (kq + 16u * k) * P::KS + 4u * w);
                    kf[k] = make_float4(fp16_bits_to_f32(kw.x & 0xFFFF), fp16_bits_to_f32(kw.x >> 16),
                                        fp16_bits_to_f32(kw.y & 0xFFFF), fp16_bits_to_f32(kw.y >> 16));
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float4 qv = *reinterpret_cast<const float4*>(qs + (4u * mq + i) * P::QS + 4u * w);
#pragma unroll
                    for (int k = 0; k < 4; ++k) s[i][k] = s[i][k] + dot4(qv, kf[k]);
                }
            }
#pragma unroll
            for (int k = 0; k < 4; ++k)
                *reinterpret_cast<float4*>(ps + (kq + 16u * k) * P::PS + 4u * mq) =
                    make_float4(s[0][k], s[1][k], s[2][k], s[3][k]);
        }
        __syncthreads();

        // 2. Each (query, tile): the top of its live scores.
        for (uint32_t i = tid; i < Q * T; i += kThreads) {
            const uint32_t m = i % Q, t = i / Q;
            const uint32_t p = q_pos[m], early = earliest_of(p, a.window);
            bool seen = false;
            float top = 0.0f;
            if (m < nq) {
                for (uint32_t b = t * B; b < (t + 1u) * B; ++b) {
                    const uint32_t j = key0 + b;
                    if (j <= p && j >= early) {
                        const float s = ps[b * P::PS + m];
                        top = seen ? fmaxf(top, s) : s;
                        seen = true;
                    }
                }
            }
            t_max[m * T + t] = top;
            t_seen[m * T + t] = seen ? 1.0f : 0.0f;
        }
        __syncthreads();

        // 3. Each query, tiles in order: the running top and each tile's alpha.
        if (tid < Q) {
            const uint32_t m = tid;
            bool live = false;
            float cm = 0.0f;
            for (uint32_t t = 0; t < T; ++t) {
                float al = 1.0f;
                if (t_seen[m * T + t] != 0.0f) {
                    const float tm = t_max[m * T + t];
                    const float old = live ? cm : tm;
                    live = true;
                    const float top = fmaxf(old, tm);
                    al = old == top ? 1.0f : exp2_np(old - top);
                    t_top[m * T + t] = top;
                    cm = top;
                }
                t_alpha[m * T + t] = al;
            }
            c_m[m] = cm;
            f_fold[m] = live ? 1.0f : 0.0f;
        }
        __syncthreads();

        // 4. Each (query, tile): the weights and their sum in key order.
        for (uint32_t i = tid; i < Q * T; i += kThreads) {
            const uint32_t m = i % Q, t = i / Q;
            const uint32_t p = q_pos[m], early = earliest_of(p, a.window);
            if (t_seen[m * T + t] != 0.0f) {
                const float top = t_top[m * T + t];
                float sum = 0.0f;
                for (uint32_t b = t * B; b < (t + 1u) * B; ++b) {
                    const uint32_t j = key0 + b;
                    float e = 0.0f;
                    if (j <= p && j >= early) e = exp2_np(ps[b * P::PS + m] - top);
                    ps[b * P::PS + m] = e;
                    sum = sum + e;
                }
                t_sum[m * T + t] = sum;
            } else {
                for (uint32_t b = t * B; b < (t + 1u) * B; ++b) ps[b * P::PS + m] = 0.0f;
            }
        }
        __syncthreads();

        // 5. Each query: the chunk's l, then the fold factors (fold_factors,
        //    :101-116) and the run's m and l (fold_sum, :118-124).
        if (tid < Q && f_fold[tid] != 0.0f) {
            const uint32_t m = tid;
            float cl = 0.0f;
            for (uint32_t t = 0; t < T; ++t)
                if (t_seen[m * T + t] != 0.0f) cl = fmaf(cl, t_alpha[m * T + t], t_sum[m * T + t]);
            const float cm = c_m[m];
            const float rm = run_m[m];
            float fa, fb, fm;
            if (run_live[m] == 0.0f) { fa = 0.0f; fb = 1.0f; fm = cm; }
            else if (rm == cm) { fa = 1.0f; fb = 1.0f; fm = rm; }
            else if (rm > cm) { fa = 1.0f; fb = exp2_np(cm - rm); fm = rm; }
            else { fa = exp2_np(rm - cm); fb = 1.0f; fm = cm; }
            run_l[m] = fmaf(run_l[m], fa, cl * fb);
            run_m[m] = fm;
            run_live[m] = 1.0f;
            f_a[m] = fa;
            f_b[m] = fb;
        }
        __syncthreads();

        // 6. P·V over the staged keys, tiles in order, then the fold into O.
        for (uint32_t task = tid; task < (Q / 4u) * (D / 8u); task += kThreads) {
            const uint32_t eq = task % (D / 8u), mq = task / (D / 8u);
            float o[4][8];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int e = 0; e < 8; ++e) o[i][e] = 0.0f;
            const uint32_t b_lo = j_lo - key0, b_hi = j_hi - key0;
            for (uint32_t t = b_lo / B; t * B < b_hi; ++t) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float al = t_alpha[(4u * mq + i) * T + t];
#pragma unroll
                    for (int e = 0; e < 8; ++e) o[i][e] = o[i][e] * al;
                }
                const uint32_t be = min((t + 1u) * B, b_hi);
                for (uint32_t b = max(t * B, b_lo); b < be; ++b) {
                    const float4 pw = *reinterpret_cast<const float4*>(ps + b * P::PS + 4u * mq);
                    const uint4 vw = *reinterpret_cast<const uint4*>(vs + b * P::VS + 8u * eq);
                    float v[8];
                    v[0] = fp16_bits_to_f32(vw.x & 0xFFFF); v[1] = fp16_bits_to_f32(vw.x >> 16);
                    v[2] = fp16_bits_to_f32(vw.y & 0xFFFF); v[3] = fp16_bits_to_f32(vw.y >> 16);
                    v[4] = fp16_bits_to_f32(vw.z & 0xFFFF); v[5] = fp16_bits_to_f32(vw.z >> 16);
                    v[6] = fp16_bits_to_f32(vw.w & 0xFFFF); v[7] = fp16_bits_to_f32(vw.w >> 16);
                    const float pv[4] = {pw.x, pw.y, pw.z, pw.w};
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        if (pv[i] != 0.0f) {
#pragma unroll
                            for (int e = 0; e < 8; ++e) o[i][e] = fmaf(pv[i], v[e], o[i][e]);
                        }
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t m = 4u * mq + i;
                if (f_fold[m] == 0.0f) continue;
                const float fa = f_a[m], fb = f_b[m];
                float4* op = reinterpret_cast<float4*>(orun + m * D + 8u * eq);
                float4 lo = op[0], hi = op[1];
                lo.x = fmaf(lo.x, fa, o[i][0] * fb); lo.y = fmaf(lo.y, fa, o[i][1] * fb);
                lo.z = fmaf(lo.z, fa, o[i][2] * fb); lo.w = fmaf(lo.w, fa, o[i][3] * fb);
                hi.x = fmaf(hi.x, fa, o[i][4] * fb); hi.y = fmaf(hi.y, fa, o[i][5] * fb);
                hi.z = fmaf(hi.z, fa, o[i][6] * fb); hi.w = fmaf(hi.w, fa, o[i][7] * fb);
                op[0] = lo;
                op[1] = hi;
            }
        }
    }
    grid_dependents_launch();
    __syncthreads();
    // out = O / l (0 for a query no key reached).
    for (uint32_t i = tid; i < nq * (D / 4u); i += kThreads) {
        const uint32_t m = i / (D / 4u), w = i % (D / 4u);
        const uint32_t r = m / G, h = kvh * G + m % G;
        float4 v = *reinterpret_cast<const float4*>(orun + m * D + 4u * w);
        if (run_live[m] != 0.0f) {
            const float l = run_l[m];
            v.x = v.x / l; v.y = v.y / l; v.z = v.z / l; v.w = v.w / l;
        } else {
            v = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        reinterpret_cast<float4*>(a.out + (static_cast<size_t>(row0 + r) * a.query_heads + h) * D)[w] = v;
    }
}

template <uint32_t D>
cudaError_t launch_prefill(const AttentionArgs& a, cudaStream_t stream, bool pdl) {
    using P = Prefill<D>;
    auto kernel = attention_prefill_kernel<D>;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(P::kSmem));
        if (e != cudaSuccess) return e;
        configured = true;
    }
    const uint32_t R = P::Q / (a.query_heads / a.kv_heads);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.kv_heads, (a.tokens + R - 1) / R);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = P::kSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, a);
}

}  // namespace

bool attention_prefill_fits(const AttentionArgs& a) {
    const uint32_t G = a.query_heads / a.kv_heads;
    const uint32_t Q = a.head_dim <= 128 ? 64u : 32u;
    return (a.head_dim == 64 || a.head_dim == 128 || a.head_dim == 256) && G >= 1 && Q % G == 0;
}

cudaError_t attention_prefill_run(const AttentionArgs& a, cudaStream_t stream, bool pdl) {
    switch (a.head_dim) {
        case 64: return launch_prefill<64>(a, stream, pdl);
        case 128: return launch_prefill<128>(a, stream, pdl);
        case 256: return launch_prefill<256>(a, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace cb
