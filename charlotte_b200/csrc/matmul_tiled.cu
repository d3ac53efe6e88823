// Prefill matrix products, Y = X·Wᵀ for a step of many tokens, with the
// reference's order of addition (plainsight-systems/charlotte,
// src/core/kernels/matmul/matmul.wgsl prefill_write/prefill_qkv/
// prefill_gated/prefill_gated_input :520-590, tile_range :410): every
// output is the same 32 range sums as the decode form's, each an fma chain
// from zero over its range's groups with k in order, added to a total from
// zero in range order. The sums are the decode form's, bit for bit, so a
// token's output does not depend on the step it came in (matmul.h:34-50).
//
// B200 mapping: a register-tiled fp32 GEMM on the CUDA cores.
//  - A CTA owns a BM-token × BN-slot tile. Each thread holds TM × 8 outputs
//    as two accumulators each: `s`, the open range's chain, and `total`.
//    K is walked one 32-weight group a step, in order; after the group that
//    closes a range, total = total + s and s restarts from zero. That is
//    exactly the reference's order, so no split over K is allowed, and the
//    tile's parallelism is all in M and N.
//  - Each group step, every weight of the tile is decoded once (the exact
//    magic-float decode of formats.cuh) into shared memory as fp32, and x is
//    staged transposed (k-major) so one 128-bit read gives a thread four
//    tokens; a float4-granular XOR swizzle by k/4 keeps both the transposing
//    stores and the reads free of bank conflicts.
//  - Double-buffered through registers: the next group's codes and x are
//    loaded while the current group is multiplied; one barrier a step.
//  - Gated products pair an output's gate row and up row in one thread (the
//    tile's first BN/2 slots are gate rows, the second BN/2 the same
//    outputs' up rows), so act(gate)·up is formed in registers.
//  - Weight codes do not depend on the previous launch: under programmatic
//    dependent launch the first group's codes are read before
//    griddepcontrol.wait; x after it.
#include <cuda_runtime.h>

#include <cstdint>
#include <utility>

#include "formats.cuh"
#include "matmul.h"
#include "numerics.cuh"
#include "tma.cuh"

namespace cb {

namespace {

// Whether group g closes a range: the range r holding g is the largest r
// with floor(r·G/32) <= g, and it closes at floor((r+1)·G/32).
__device__ __forceinline__ bool closes_range(uint32_t g, uint32_t G) {
    const uint32_t r = (32u * (g + 1u) + G - 1u) / G - 1u;
    return (r + 1u) * G / 32u == g + 1u;
}

template <int BM_, int BN_, int TM_>
struct Tile {
    static constexpr int BM = BM_, BN = BN_, TM = TM_, TN = 8;
    static constexpr int kThreads = (BM / TM) * (BN / TN);
    static constexpr int kParts = kThreads / BN;                 // threads decoding one slot's group
    static constexpr int kPartWeights = 32 / kParts;
    static constexpr int kXVec = BM * 8 / kThreads;              // float4 of x a thread stages a step
    static constexpr size_t kSmem = 2ull * 32u * (BM + BN) * 4u;
    // The 256-thread four-row tile is the occupancy shape: held to 128
    // registers a thread, two of its CTAs share an SM.
    static constexpr int kMinBlocks = TM == 4 && kThreads == 256 ? 2 : 1;
    static_assert(kThreads % BN == 0 && (kParts == 1 || kParts == 2), "one or two threads a slot");
    static_assert(BM * 8 % kThreads == 0, "x staging divides evenly");
    static_assert(BM >= 32 && (BM / 4) % 8 == 0, "x swizzle spans eight float4 columns");
    static_assert(TM == 4 || TM == 8, "");
};

// Index of token t, weight k in the transposed x stage: float4 column t/4
// XOR'd with k/4 (mod 8).
template <int BM>
__device__ __forceinline__ uint32_t xs_index(uint32_t k, uint32_t t) {
    return k * BM + 4u * ((t >> 2) ^ ((k >> 2) & 7u)) + (t & 3u);
}

// Decodes weights [K0, K0 + sizeof...(ks)) of a group into column j of the
// weight stage (k-major, BN floats a row).
template <typename F, int BN, int K0, int... ks>
__device__ __forceinline__ void decode_part(const F& f, float* ws_col, std::integer_sequence<int, ks...>) {
    const typename F::Consts c = f.consts();
    ((ws_col[(K0 + ks) * BN] = F::template weight<K0 + ks>(f, c)), ...);
}

template <typename F, typename T>
__global__ void __launch_bounds__(T::kThreads, T::kMinBlocks) tiled_kernel(const MatmulArgs a) {
    constexpr int BM = T::BM, BN = T::BN, TM = T::TM;
    extern __shared__ __align__(16) float smem_f[];
    float* xs = smem_f;                 // [2][32][BM], swizzled
    float* ws = smem_f + 2 * 32 * BM;   // [2][32][BN]

    const uint32_t G = a.columns / 32u;
    const uint32_t tid = threadIdx.x;
    const bool gated = a.epilogue == kGated;
    const uint32_t m0 = blockIdx.x * BM;
    // Split form: this CTA's groups are range blockIdx.z's alone.
    const bool split = a.range_sums != nullptr;
    const uint32_t g_lo = split ? blockIdx.z * G / 32u : 0u, g_hi = split ? (blockIdx.z + 1u) * G / 32u : G;
    const uint32_t n0 = blockIdx.y * (gated ? BN / 2 : BN);   // first slot (gated: first output)

    // ---- decode role: slot j of the tile, weights of part p --------------
    // (members are picked by value with unrolled compares: a kernel
    // parameter indexed at run time would be copied to local memory)
    const uint32_t j = tid % BN, part = tid / BN;
    const uint8_t* sp[F::kStreams];
    bool live = false;
    {
        int q = -1;
        uint32_t row = 0;
        if (gated) {
            const uint32_t o = n0 + (j < BN / 2 ? j : j - BN / 2);
            if (o < a.member[0].rows) {
                q = j < BN / 2 ? 0 : 1;
                row = (q == 0 ? a.member[0].first_row : a.member[1].first_row) + o;
            }
        } else {
            uint32_t n = n0 + j;
#pragma unroll
            for (int i = 0; i < 3; ++i) {
                if (q < 0 && i < static_cast<int>(a.members)) {
                    if (n < a.member[i].rows) {
                        q = i;
                        row = a.member[i].first_row + n;
                    } else {
                        n -= a.member[i].rows;
                    }
                }
            }
        }
        live = q >= 0;
        const uint8_t* piece = q == 1 ? a.member[1].piece : (q == 2 ? a.member[2].piece : a.member[0].piece);
        const uint32_t blocks = q == 1 ? a.member[1].blocks : (q == 2 ? a.member[2].blocks : a.member[0].blocks);
#pragma unroll
        for (int s = 0; s < F::kStreams; ++s)
            sp[s] = piece + RowStreams<F>::base(s, blocks) +
                    static_cast<uint64_t>(live ? row : 0u) * RowStreams<F>::row_bytes(s, G);
    }

    // ---- x role: float4 v = it·threads + tid is token v/8, k 4·(v%8) -------
    // x comes through L2 (ld.global.cg), never the non-coherent read-only
    // path: under programmatic dependent launch this grid starts while the
    // launch that writes x is still running.
    float4 xr[T::kXVec];
    auto load_x = [&](uint32_t g) {
#pragma unroll
        for (int it = 0; it < T::kXVec; ++it) {
            const uint32_t v = it * T::kThreads + tid;
            const uint32_t t = m0 + v / 8u;
            xr[it] = t < a.tokens
                         ? __ldcg(reinterpret_cast<const float4*>(a.x + static_cast<size_t>(t) * a.x_stride + g * 32u) +
                                  (v % 8u))
                         : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    auto store_x = [&](float* dst) {
#pragma unroll
        for (int it = 0; it < T::kXVec; ++it) {
            const uint32_t v = it * T::kThreads + tid;
            const uint32_t t = v / 8u, k = 4u * (v % 8u);
            dst[xs_index<BM>(k + 0, t)] = xr[it].x;
            dst[xs_index<BM>(k + 1, t)] = xr[it].y;
            dst[xs_index<BM>(k + 2, t)] = xr[it].z;
            dst[xs_index<BM>(k + 3, t)] = xr[it].w;
        }
    };
    F raw;
    auto load_w = [&](uint32_t g) {
        if (live) raw.load(sp, g);
        else raw.zero();
    };
    auto store_w = [&](float* dst) {
        if (T::kParts == 1 || part == 0)
            decode_part<F, BN, 0>(raw, dst + j, std::make_integer_sequence<int, T::kPartWeights>{});
        else
            decode_part<F, BN, T::kPartWeights>(raw, dst + j, std::make_integer_sequence<int, T::kPartWeights>{});
    };

    // ---- compute role: tokens ty·4.. (+BM/2), slots tx·4.. and BN/2 + tx·4.. --
    const uint32_t tx = tid % (BN / 8), ty = tid / (BN / 8);
    // Outputs (i, 2p) and (i, 2p + 1) as one pair: the paired FMA
    // (fma.rn.f32x2) rounds each half once, so each output keeps fmaf's bits.
    float2 s[TM][4], total[TM][4];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int p = 0; p < 4; ++p) { s[i][p] = make_float2(0.0f, 0.0f); total[i][p] = make_float2(0.0f, 0.0f); }

    if (g_lo < g_hi) load_w(g_lo);
    grid_dependency_wait();
    if (g_lo < g_hi) {
        load_x(g_lo);
        store_w(ws);
        store_x(xs);
    }
    __syncthreads();

    for (uint32_t g = g_lo; g < g_hi; ++g) {
        const uint32_t buf = (g - g_lo) & 1u;
        const bool more = g + 1u < g_hi;
        if (more) {
            load_w(g + 1u);
            load_x(g + 1u);
        }
        const float* xb = xs + buf * 32u * BM;
        const float* wb = ws + buf * 32u * BN;
#pragma unroll
        for (uint32_t k = 0; k < 32; ++k) {
            float xv[TM];
            const uint32_t sw = (k >> 2) & 7u;
            const float4 x0 = *reinterpret_cast<const float4*>(xb + k * BM + 4u * (ty ^ sw));
            xv[0] = x0.x; xv[1] = x0.y; xv[2] = x0.z; xv[3] = x0.w;
            if constexpr (TM == 8) {
                const float4 x1 = *reinterpret_cast<const float4*>(xb + k * BM + 4u * ((ty + BM / 8) ^ sw));
                xv[4] = x1.x; xv[5] = x1.y; xv[6] = x1.z; xv[7] = x1.w;
            }
            const float4 w0 = *reinterpret_cast<const float4*>(wb + k * BN + 4u * tx);
            const float4 w1 = *reinterpret_cast<const float4*>(wb + k * BN + BN / 2 + 4u * tx);
            const float2 wp[4] = {make_float2(w0.x, w0.y), make_float2(w0.z, w0.w), make_float2(w1.x, w1.y),
                                  make_float2(w1.z, w1.w)};
#pragma unroll
            for (int i = 0; i < TM; ++i) {
                const float2 xx = make_float2(xv[i], xv[i]);
#pragma unroll
                for (int p = 0; p < 4; ++p) s[i][p] = __ffma2_rn(wp[p], xx, s[i][p]);
            }
        }
        if (!split && closes_range(g, G)) {
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int p = 0; p < 4; ++p) { total[i][p] = __fadd2_rn(total[i][p], s[i][p]); s[i][p] = make_float2(0.0f, 0.0f); }
        }
        if (more) {
            store_w(ws + (buf ^ 1u) * 32u * BN);
            store_x(xs + (buf ^ 1u) * 32u * BM);
        }
        __syncthreads();
    }
    grid_dependents_launch();

    // ---- epilogue -----------------------------------------------------------
    if (split) {
        // The range's sums of every product row of the tile (an empty
        // range's zeros, which the combine adds as the reference does).
#pragma unroll
        for (int i = 0; i < TM; ++i) {
            const uint32_t t = m0 + (i < 4 ? ty * 4u + i : BM / 2 + ty * 4u + (i - 4));
            if (t >= a.tokens) continue;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const uint32_t n = n0 + (c < 4 ? tx * 4u + c : BN / 2 + tx * 4u + (c - 4));
                if (n < a.total_rows)
                    a.range_sums[(static_cast<size_t>(blockIdx.z) * a.tokens + t) * a.total_rows + n] =
                        (c & 1) ? s[i][c >> 1].y : s[i][c >> 1].x;
            }
        }
        return;
    }
    auto sum = [&](int i, int c) { return (c & 1) ? total[i][c >> 1].y : total[i][c >> 1].x; };
#pragma unroll
    for (int i = 0; i < TM; ++i) {
        const uint32_t t = m0 + (i < 4 ? ty * 4u + i : BM / 2 + ty * 4u + (i - 4));
        if (t >= a.tokens) continue;
        if (gated) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint32_t o = n0 + tx * 4u + c;
                if (o < a.member[0].rows)
                    a.out[0][static_cast<size_t>(t) * a.out_stride[0] + a.member[0].out_offset + o] =
                        activate(a.activation, sum(i, c)) * sum(i, 4 + c);
            }
            continue;
        }
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            uint32_t n = n0 + (c < 4 ? tx * 4u + c : BN / 2 + tx * 4u + (c - 4));
            int q = -1;
#pragma unroll
            for (int m = 0; m < 3; ++m) {
                if (q < 0 && m < static_cast<int>(a.members)) {
                    if (n < a.member[m].rows) q = m;
                    else n -= a.member[m].rows;
                }
            }
            if (q < 0) continue;
            const uint32_t o =
                (q == 1 ? a.member[1].out_offset : (q == 2 ? a.member[2].out_offset : a.member[0].out_offset)) + n;
            if (a.epilogue == kQKV) {
                float* out = q == 1 ? a.out[1] : (q == 2 ? a.out[2] : a.out[0]);
                const uint32_t stride = q == 1 ? a.out_stride[1] : (q == 2 ? a.out_stride[2] : a.out_stride[0]);
                out[static_cast<size_t>(t) * stride + o] = sum(i, c);
            } else if (a.epilogue == kWrite) {
                a.out[0][static_cast<size_t>(t) * a.out_stride[0] + o] = sum(i, c);
            } else {   // kGatedByInput (matmul.wgsl:346-350)
                const float u = a.gate_input[static_cast<size_t>(a.token + t) * a.gate_input_stride +
                                             a.gate_input_column + o];
                a.out[0][static_cast<size_t>(t) * a.out_stride[0] + o] = activate(a.activation, sum(i, c)) * u;
            }
        }
    }
}

template <typename F, typename T>
cudaError_t launch_tiled(const MatmulArgs& a, cudaStream_t stream, bool pdl) {
    auto kernel = tiled_kernel<F, T>;
    static bool configured = false;   // per instantiation
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(T::kSmem));
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    const bool gated = a.epilogue == kGated;
    const uint32_t slots = gated ? a.member[0].rows : a.total_rows;
    const uint32_t per_tile = gated ? T::BN / 2 : T::BN;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((a.tokens + T::BM - 1) / T::BM, (slots + per_tile - 1) / per_tile, a.range_sums ? 32u : 1u);
    cfg.blockDim = dim3(T::kThreads);
    cfg.dynamicSmemBytes = T::kSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, a);
}

using TileL = Tile<128, 128, 8>;   // 256 threads, 64 outputs each
using TileM = Tile<64, 128, 8>;    // 128 threads
using TileW = Tile<64, 128, 4>;    // 256 threads, 32 outputs each: more warps for few tiles
using TileS = Tile<32, 128, 4>;    // 128 threads: short steps
using TileT = Tile<32, 64, 4>;     // 64 threads: short steps of narrow products

// A rough figure of merit of a tile shape for this product: the warps it
// puts on the SMs (up to eight an SM), times the share of its tile rows that
// are real tokens, times a per-thread efficiency (fewer outputs a thread
// read more shared memory a multiply).
template <typename T>
double merit(const MatmulArgs& a, int sm_count) {
    const bool gated = a.epilogue == kGated;
    const uint32_t slots = gated ? a.member[0].rows : a.total_rows;
    const uint32_t per_tile = gated ? T::BN / 2 : T::BN;
    const double mt = (a.tokens + T::BM - 1) / T::BM, nt = (slots + per_tile - 1) / per_tile;
    const double warps = mt * nt * (T::kThreads / 32) * (a.range_sums ? 32.0 : 1.0);
    const double want = 8.0 * sm_count;
    const double fill = warps >= want ? 1.0 : warps / want;
    const double used = static_cast<double>(a.tokens) / (mt * T::BM);
    const double per_thread = T::TM == 8 ? 1.0 : 0.8;
    return fill * used * per_thread;
}

template <typename F>
cudaError_t dispatch_tiled(const MatmulArgs& a, int sm_count, cudaStream_t stream, bool pdl) {
    const double mL = merit<TileL>(a, sm_count), mM = merit<TileM>(a, sm_count), mW = merit<TileW>(a, sm_count),
                 mS = merit<TileS>(a, sm_count), mT = merit<TileT>(a, sm_count);
    double best = mL;
    int pick = 0;
    if (mM > best * 1.05) { best = mM; pick = 1; }
    if (mW > best * 1.05) { best = mW; pick = 2; }
    if (mS > best * 1.05) { best = mS; pick = 3; }
    if (mT > best * 1.05) { best = mT; pick = 4; }
    switch (pick) {
        case 0: return launch_tiled<F, TileL>(a, stream, pdl);
        case 1: return launch_tiled<F, TileM>(a, stream, pdl);
        case 2: return launch_tiled<F, TileW>(a, stream, pdl);
        case 3: return launch_tiled<F, TileS>(a, stream, pdl);
        default: return launch_tiled<F, TileT>(a, stream, pdl);
    }
}

// The split form's combine (combine_write, combine_qkv, combine_gated_input,
// matmul.wgsl:651-695): product row p of token t is the 32 range sums added
// to a total from zero in range order, then the epilogue.
__global__ void __launch_bounds__(256) combine_kernel(const MatmulArgs a) {
    grid_dependency_wait();
    const uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < static_cast<uint64_t>(a.tokens) * a.total_rows) {
        const uint32_t t = static_cast<uint32_t>(i / a.total_rows), p = static_cast<uint32_t>(i % a.total_rows);
        const size_t plane = static_cast<size_t>(a.tokens) * a.total_rows;
        const float* rs = a.range_sums + static_cast<size_t>(t) * a.total_rows + p;
        float v[32];
#pragma unroll
        for (int r = 0; r < 32; ++r) v[r] = __ldcg(rs + r * plane);
        float total = 0.0f;
#pragma unroll
        for (int r = 0; r < 32; ++r) total = total + v[r];
        uint32_t n = p;
        int q = 0;
        if (a.members > 1 && n >= a.member[0].rows) {
            n -= a.member[0].rows;
            q = 1;
            if (a.members > 2 && n >= a.member[1].rows) {
                n -= a.member[1].rows;
                q = 2;
            }
        }
        const uint32_t o =
            (q == 1 ? a.member[1].out_offset : (q == 2 ? a.member[2].out_offset : a.member[0].out_offset)) + n;
        if (a.epilogue == kQKV) {
            float* out = q == 1 ? a.out[1] : (q == 2 ? a.out[2] : a.out[0]);
            const uint32_t stride = q == 1 ? a.out_stride[1] : (q == 2 ? a.out_stride[2] : a.out_stride[0]);
            out[static_cast<size_t>(t) * stride + o] = total;
        } else if (a.epilogue == kWrite) {
            a.out[0][static_cast<size_t>(t) * a.out_stride[0] + o] = total;
        } else {
            const float u =
                a.gate_input[static_cast<size_t>(a.token + t) * a.gate_input_stride + a.gate_input_column + o];
            a.out[0][static_cast<size_t>(t) * a.out_stride[0] + o] = activate(a.activation, total) * u;
        }
    }
    grid_dependents_launch();
}

cudaError_t launch_combine(const MatmulArgs& a, cudaStream_t stream, bool pdl) {
    const uint64_t n = static_cast<uint64_t>(a.tokens) * a.total_rows;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<uint32_t>((n + 255) / 256));
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, combine_kernel, a);
}

}  // namespace

// Measured on B200 (bench.py --case split-forms, Q4_0, K of 2,048 to 8,192,
// 1,024 to 2,048 rows, 4 to 512 tokens): the split form is the fastest exact
// form from 24–32 tokens while the tiled form's 128 × 128 tiles would fill
// at most half the SMs (Gemma's down at 64 tokens 28.6 µs against 70.3
// streamed and 501 tiled; Llama's down at 512 tokens 458 against 592
// tiled); below ~24 tokens the streamed form wins (4 to 16 tokens: 4–47 µs
// against 8–38).
bool split_form(uint32_t tokens, uint32_t slots, uint32_t columns, uint32_t epilogue, int sm_count) {
    if (epilogue == kGated || columns / 32u < 64u || tokens < 24u) return false;
    const uint64_t tiles = static_cast<uint64_t>((tokens + 127u) / 128u) * ((slots + 127u) / 128u);
    return tiles * 2u <= static_cast<uint64_t>(sm_count);
}

cudaError_t matmul_split(const MatmulArgs& a, int sm_count, cudaStream_t stream, bool pdl) {
    if (!a.range_sums || a.epilogue == kGated) return cudaErrorInvalidValue;
    if (cudaError_t e = matmul_tiled(a, sm_count, stream, pdl); e != cudaSuccess) return e;
    return launch_combine(a, stream, pdl);
}

cudaError_t matmul_tiled(const MatmulArgs& a, int sm_count, cudaStream_t stream, bool pdl) {
    switch (a.format) {
        case kQ4_0: return dispatch_tiled<Q4_0>(a, sm_count, stream, pdl);
        case kQ8_0: return dispatch_tiled<Q8_0>(a, sm_count, stream, pdl);
        case kQ6_K: return dispatch_tiled<Q6_K>(a, sm_count, stream, pdl);
        case kQ4_1: return dispatch_tiled<Q4_1>(a, sm_count, stream, pdl);
        case kBF16: return dispatch_tiled<BF16>(a, sm_count, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace cb
