// Attention for prefill steps on the tensor cores — the tolerance tier
// (CB_RUN_TENSOR; the decoder's CB_DECODER_TENSOR_PREFILL): the same
// attention as attention.wgsl main :138-360 (causal, the layer's window,
// scale·log2e, softmax in log2 units), but with the operands rounded to f16
// and the products summed by the tensor cores in their own order, so not
// the reference's bits: outputs within the tolerance the tensor-form
// products keep (tests/test_attention_tensor_gpu.py states it).
//
// B200 mapping (flash attention, one pass): a CTA per (kv head, block of
// query positions); a warp per (16 positions, one of the kv head's G query
// heads), so the kv head's keys and values are staged once for all G heads.
// Each 64-key tile comes into shared memory by cp.async (double-buffered,
// rows padded by 16 bytes so ldmatrix reads are conflict-free); S = Q·Kᵀ by
// mma.sync m16n8k16 (f16 in, f32 out) with the query fragments held in
// registers (q·scale·log2e rounded to f16 once); the online softmax in
// registers (row max and sum across the quad, exp2); P, rounded to f16, is
// the A fragment of P·V straight from S's accumulator layout; V's fragments
// by ldmatrix.trans. Keys past a query's position or before its window
// weigh nothing. O / l at the end.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "api_common.h"
#include "kernels.h"
#include "tma.cuh"

namespace cb {

namespace {

constexpr uint32_t kKeys = 64;   // keys a tile
constexpr float kNegInf = -__builtin_huge_valf();

__device__ __forceinline__ uint32_t earliest(uint32_t p, uint32_t window) { return p + 1u > window ? p + 1u - window : 0u; }

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldmatrix_x2(uint32_t& r0, uint32_t& r1, const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n" : "=r"(r0), "=r"(r1) : "r"(smem_addr(p)));
}

__device__ __forceinline__ void ldmatrix_x2_trans(uint32_t& r0, uint32_t& r1, const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];\n"
                 : "=r"(r0), "=r"(r1)
                 : "r"(smem_addr(p)));
}

__device__ __forceinline__ void cp_async16_zfill(void* dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_addr(dst)), "l"(src),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

template <uint32_t D>
struct TensorAttention {
    static constexpr uint32_t kRow = D + 8;                    // halves a staged row (16-byte pad)
    static constexpr uint32_t kTile = kKeys * kRow;            // halves a K or V tile
    static constexpr size_t kSmem = 2ull * 2 * kTile * 2;      // K and V, two stages
};

// Warps = G·WQ: warp w is head w % G of the kv head, positions
// 16·(w / G) .. +15 of the CTA's block of 16·WQ positions.
template <uint32_t D>
__global__ void __launch_bounds__(256) attention_tensor_kernel(const AttentionArgs a, uint32_t WQ) {
    using TA = TensorAttention<D>;
    extern __shared__ __align__(16) uint16_t sm16[];
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t G = a.query_heads / a.kv_heads;
    const uint32_t kvh = blockIdx.x;
    const uint32_t head = kvh * G + warp % G;
    const uint32_t block_rows = 16u * WQ;
    // the longest blocks (latest rows, most keys) start first
    const uint32_t row0 = (gridDim.y - 1u - blockIdx.y) * block_rows;   // the CTA's first row of the step
    const uint32_t wrow0 = row0 + 16u * (warp / G);                // this warp's first row
    const uint32_t threads = blockDim.x;
    const uint32_t pos0 = a.position ? *a.position : a.position0;
    grid_dependency_wait();

    // The CTA's key range: from the first row's earliest key to its last row.
    const uint32_t last_row = min(row0 + block_rows, a.tokens) - 1u;
    const uint32_t key_lo = earliest(pos0 + row0, a.window) / kKeys * kKeys;
    const uint32_t key_hi = pos0 + last_row;   // inclusive
    const uint32_t tiles = (key_hi - key_lo) / kKeys + 1u;

    // stage s: keys at sm16 + s·tile, values at sm16 + (2 + s)·tile
    auto kst = [&](uint32_t s) { return sm16 + s * TA::kTile; };
    auto vst = [&](uint32_t s) { return sm16 + (2u + s) * TA::kTile; };
    auto load_tile = [&](uint32_t t, uint32_t s) {
        const uint32_t k0 = key_lo + t * kKeys;
        constexpr uint32_t chunks = D / 8;   // 16-byte chunks a row
        for (uint32_t i = threadIdx.x; i < kKeys * chunks; i += threads) {
            const uint32_t r = i / chunks, c = i % chunks;
            const uint32_t j = k0 + r;
            const bool valid = j <= key_hi;
            const size_t at = (static_cast<size_t>((valid ? j : key_lo) % a.slots) * a.kv_heads + kvh) * D + c * 8u;
            cp_async16_zfill(kst(s) + r * TA::kRow + c * 8u, a.key_cache + at, valid);
            cp_async16_zfill(vst(s) + r * TA::kRow + c * 8u, a.value_cache + at, valid);
        }
        cp_async_commit();
    };
    load_tile(0, 0);

    // The warp's query fragments: rows g and g+8 of its 16 positions, q·scale·log2e in f16.
    const uint32_t g = lane / 4u, c = lane % 4u;
    uint32_t qf[D / 16][4];
    {
        const uint32_t ra = wrow0 + g, rb = wrow0 + g + 8u;
        const float* qa = a.query + (static_cast<size_t>(ra) * a.query_heads + head) * D;
        const float* qb = a.query + (static_cast<size_t>(rb) * a.query_heads + head) * D;
        const bool va = ra < a.tokens, vb = rb < a.tokens;
#pragma unroll
        for (uint32_t kk = 0; kk < D / 16; ++kk) {
            const uint32_t d0 = kk * 16u + 2u * c;
            const float2 a0 = va ? *reinterpret_cast<const float2*>(qa + d0) : make_float2(0.f, 0.f);
            const float2 a1 = vb ? *reinterpret_cast<const float2*>(qb + d0) : make_float2(0.f, 0.f);
            const float2 a2 = va ? *reinterpret_cast<const float2*>(qa + d0 + 8u) : make_float2(0.f, 0.f);
            const float2 a3 = vb ? *reinterpret_cast<const float2*>(qb + d0 + 8u) : make_float2(0.f, 0.f);
            const float s = a.scale_log2e;
            qf[kk][0] = pack_half2(a0.x * s, a0.y * s);
            qf[kk][1] = pack_half2(a1.x * s, a1.y * s);
            qf[kk][2] = pack_half2(a2.x * s, a2.y * s);
            qf[kk][3] = pack_half2(a3.x * s, a3.y * s);
        }
    }
    const uint32_t pa = pos0 + wrow0 + g, pb = pa + 8u;   // positions of rows g and g+8
    const uint32_t ea = earliest(pa, a.window), eb = earliest(pb, a.window);

    float o[D / 8][4];
#pragma unroll
    for (uint32_t n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    float m_a = kNegInf, m_b = kNegInf, l_a = 0.0f, l_b = 0.0f;

    for (uint32_t t = 0; t < tiles; ++t) {
        const uint32_t s = t & 1u;
        if (t + 1u < tiles) {
            load_tile(t + 1u, s ^ 1u);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const uint32_t k0 = key_lo + t * kKeys;
        // the warp's rows see keys up to its last position; a tile past it
        // (other warps' later rows) contributes nothing
        if (k0 <= pos0 + wrow0 + 15u) {
            float sacc[kKeys / 8][4];
#pragma unroll
            for (uint32_t n = 0; n < kKeys / 8; ++n) sacc[n][0] = sacc[n][1] = sacc[n][2] = sacc[n][3] = 0.0f;
#pragma unroll
            for (uint32_t n = 0; n < kKeys / 8; ++n) {
#pragma unroll
                for (uint32_t kk = 0; kk < D / 16; ++kk) {
                    uint32_t b0, b1;
                    const uint16_t* p = kst(s) + (n * 8u + (lane % 8u)) * TA::kRow + kk * 16u + ((lane / 8u) % 2u) * 8u;
                    ldmatrix_x2(b0, b1, p);
                    mma16816(sacc[n], qf[kk], b0, b1);
                }
            }
            // mask, row maxima
            float mx_a = kNegInf, mx_b = kNegInf;
#pragma unroll
            for (uint32_t n = 0; n < kKeys / 8; ++n) {
#pragma unroll
                for (uint32_t e = 0; e < 2; ++e) {
                    const uint32_t j = k0 + n * 8u + 2u * c + e;
                    if (!(j <= pa && j >= ea)) sacc[n][e] = kNegInf;
                    if (!(j <= pb && j >= eb)) sacc[n][2 + e] = kNegInf;
                    mx_a = fmaxf(mx_a, sacc[n][e]);
                    mx_b = fmaxf(mx_b, sacc[n][2 + e]);
                }
            }
#pragma unroll
            for (int off = 1; off <= 2; off <<= 1) {
                mx_a = fmaxf(mx_a, __shfl_xor_sync(0xFFFFFFFFu, mx_a, off));
                mx_b = fmaxf(mx_b, __shfl_xor_sync(0xFFFFFFFFu, mx_b, off));
            }
            const float nm_a = fmaxf(m_a, mx_a), nm_b = fmaxf(m_b, mx_b);
            // rows with no live key yet keep their (empty) state
            const float base_a = nm_a == kNegInf ? 0.0f : nm_a, base_b = nm_b == kNegInf ? 0.0f : nm_b;
            const float al_a = exp2f(m_a - base_a), al_b = exp2f(m_b - base_b);
            m_a = nm_a;
            m_b = nm_b;
            float sum_a = 0.0f, sum_b = 0.0f;
            uint32_t pf[kKeys / 16][4];
#pragma unroll
            for (uint32_t n = 0; n < kKeys / 8; ++n) {
                const float p0 = exp2f(sacc[n][0] - base_a), p1 = exp2f(sacc[n][1] - base_a);
                const float p2 = exp2f(sacc[n][2] - base_b), p3 = exp2f(sacc[n][3] - base_b);
                sum_a += p0 + p1;
                sum_b += p2 + p3;
                pf[n / 2][(n % 2) * 2 + 0] = pack_half2(p0, p1);
                pf[n / 2][(n % 2) * 2 + 1] = pack_half2(p2, p3);
            }
#pragma unroll
            for (int off = 1; off <= 2; off <<= 1) {
                sum_a += __shfl_xor_sync(0xFFFFFFFFu, sum_a, off);
                sum_b += __shfl_xor_sync(0xFFFFFFFFu, sum_b, off);
            }
            l_a = l_a * al_a + sum_a;
            l_b = l_b * al_b + sum_b;
#pragma unroll
            for (uint32_t n = 0; n < D / 8; ++n) {
                o[n][0] *= al_a;
                o[n][1] *= al_a;
                o[n][2] *= al_b;
                o[n][3] *= al_b;
            }
            // P·V: A = P (keys 16kk..16kk+15), B = V rows of those keys, dims 8n..8n+7
#pragma unroll
            for (uint32_t kk = 0; kk < kKeys / 16; ++kk) {
                const uint32_t af[4] = {pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3]};
#pragma unroll
                for (uint32_t n = 0; n < D / 8; ++n) {
                    uint32_t b0, b1;
                    const uint16_t* p = vst(s) + (kk * 16u + (lane % 16u)) * TA::kRow + n * 8u;
                    ldmatrix_x2_trans(b0, b1, p);
                    mma16816(o[n], af, b0, b1);
                }
            }
        }
        __syncthreads();   // the stage is read before the next tile's copies land in it
    }
    grid_dependents_launch();
    const uint32_t ra = wrow0 + g, rb = ra + 8u;
    const float ia = l_a > 0.0f ? 1.0f / l_a : 0.0f, ib = l_b > 0.0f ? 1.0f / l_b : 0.0f;
#pragma unroll
    for (uint32_t n = 0; n < D / 8; ++n) {
        const uint32_t d0 = n * 8u + 2u * c;
        const size_t at_a = (static_cast<size_t>(ra) * a.query_heads + head) * D + d0;
        const size_t at_b = (static_cast<size_t>(rb) * a.query_heads + head) * D + d0;
        if (ra < a.tokens) {
            *reinterpret_cast<float2*>(a.out + at_a) = make_float2(o[n][0] * ia, o[n][1] * ia);
            if (a.out16) *reinterpret_cast<__half2*>(static_cast<__half*>(a.out16) + at_a) =
                             __floats2half2_rn(o[n][0] * ia, o[n][1] * ia);
        }
        if (rb < a.tokens) {
            *reinterpret_cast<float2*>(a.out + at_b) = make_float2(o[n][2] * ib, o[n][3] * ib);
            if (a.out16) *reinterpret_cast<__half2*>(static_cast<__half*>(a.out16) + at_b) =
                             __floats2half2_rn(o[n][2] * ib, o[n][3] * ib);
        }
    }
}

template <uint32_t D>
cudaError_t launch_tensor_attention(const AttentionArgs& a, cudaStream_t stream, bool pdl) {
    using TA = TensorAttention<D>;
    auto kernel = attention_tensor_kernel<D>;
    static bool configured = false;
    if (!configured) {
        const cudaError_t e =
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(TA::kSmem));
        if (e != cudaSuccess) return e;
        configured = true;
    }
    const uint32_t G = a.query_heads / a.kv_heads;
    // Warps a CTA: G·WQ, up to 8; fewer row blocks a CTA while the grid is
    // under two CTAs an SM (the causal triangle makes the late blocks long:
    // more, shorter CTAs balance it).
    const int sms = sm_count();
    const uint32_t want = 2u * (sms > 0 ? static_cast<uint32_t>(sms) : 148u);
    uint32_t WQ = G >= 8u ? 1u : 8u / G;
    while (WQ > 1u && a.kv_heads * ((a.tokens + 16u * WQ - 1u) / (16u * WQ)) < want) WQ /= 2u;
    const uint32_t block_rows = 16u * WQ;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.kv_heads, (a.tokens + block_rows - 1) / block_rows);
    cfg.blockDim = dim3(32u * G * WQ);
    cfg.dynamicSmemBytes = TA::kSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, a, WQ);
}

}  // namespace

bool attention_tensor_fits(const AttentionArgs& a) {
    const uint32_t G = a.query_heads / a.kv_heads;
    return !a.rows_are_sequences && a.tokens >= 16u && (a.head_dim == 64 || a.head_dim == 128) && G >= 1 && G <= 8 &&
           (G & (G - 1)) == 0;
}

cudaError_t attention_tensor_run(const AttentionArgs& a, cudaStream_t stream, bool pdl) {
    switch (a.head_dim) {
        case 64: return launch_tensor_attention<64>(a, stream, pdl);
        case 128: return launch_tensor_attention<128>(a, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace cb
