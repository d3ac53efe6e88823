// The decode step fused into one persistent launch: the embedding gather
// and every layer's launches of the reference's graph (plainsight-systems/
// charlotte, src/core/graph/graph.cpp: embed :155, attention :159-230,
// gated_feed_forward :232-262; the final norm of output :264-292), for one
// token at the step's position, with the same arithmetic as the separate
// kernels — each output's bits are theirs (norm.wgsl's tree, rope.wgsl's
// head tree and turns, attention.wgsl's chunks and fold, matmul.wgsl's
// ranges) — so the fused and the separate step agree bit for bit.
//
// Why: a separate decode step is ~229 small dependent launches, each paying
// microseconds of launch and drain; here the dependencies become grid-wide
// barriers between stages, and the weight rows a warp streams in its next
// product are put in flight (bulk copies into its shared stage) before it
// waits at the barrier, since weights do not depend on the step.
//
// One CTA an SM (a cooperative launch: all CTAs resident), 8 or 16 warps.
// Stages of a layer, a barrier after each:
//   A  attention norm (every CTA computes it; CTA 0 writes the residual
//      stream's next buffer) into the CTA's x stage; QKV product;
//   B  (kv head, 64-key chunk) items over the CTAs: QK-norm and rope of the
//      head's queries (and of its key and value, into the cache, for the
//      chunk holding the position), the chunk's online softmax state;
//   C  the chunks folded in order, each (query head, dimension) a thread;
//   D  O product;
//   E  feed-forward norm with the residual add; gate|up product;
//   F  down product.
// The final norm (last token) closes the launch; the head, selection and
// draw follow as separate launches.
//
// Every barrier wait is bounded: one that runs out sets the fault word and
// the launch returns (after its own bulk copies land), so the step reports
// a failure instead of hanging.
#include <cuda_runtime.h>

#include <cstdint>
#include <utility>

#include "api_common.h"
#include "decode_fused.h"
#include "formats.cuh"
#include "gemv_common.cuh"
#include "kernels.h"
#include "numerics.cuh"
#include "tma.cuh"

namespace cb {

namespace {

constexpr uint32_t kChunkF = 64;
constexpr uint32_t kFaultBarrier = 4u;

__device__ __forceinline__ uint32_t ld_acquire(const unsigned int* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release(unsigned int* p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Grid-wide barrier over `n` resident CTAs: bar[0] counts arrivals, bar[1]
// is the generation the last arrival advances. Bounded: false (fault word
// set) when the generation did not move in time.
__device__ bool grid_barrier(unsigned int* bar, uint32_t n, unsigned int* fault) {
    __shared__ int ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        ok = 1;
        const uint32_t g = ld_acquire(bar + 1);
        __threadfence();
        const uint32_t arrived = atomicAdd(bar, 1u) + 1u;
        if (arrived == n) {
            atomicExch(bar, 0u);
            __threadfence();
            st_release(bar + 1, g + 1u);
        } else {
            uint32_t i = 0;
            while (ld_acquire(bar + 1) == g) {
                if (++i > kSpinLimit) {
                    atomicOr(fault, kFaultBarrier);
                    ok = 0;
                    break;
                }
                __nanosleep(64);
            }
        }
        __threadfence();
    }
    __syncthreads();
    return ok != 0;
}

__device__ __forceinline__ uint32_t earliest_f(uint32_t p, uint32_t window) {
    return p + 1u > window ? p + 1u - window : 0u;
}

// ---- per-warp GEMV state --------------------------------------------------------
struct Warp {
    uint64_t* bars;       // 2 mbarriers, the ring's slots
    float* red;           // R rows of range sums
    uint8_t* stages;      // 2 slots of stage_bytes
    uint32_t stage_bytes;
    uint32_t it;          // slot uses so far (slot it & 1, parity (it >> 1) & 1)
    uint32_t gw, nw;      // this warp's index among all the grid's warps, and their number
};

// Puts this warp's first two batches of product p in flight.
template <typename F, int R>
__device__ void prefetch_product(const MatmulArgs& p, Warp& w, uint32_t lane) {
    const uint32_t G = p.columns / 32u;
    const uint32_t batches = batch_count<R>(p);
    for (uint32_t i = 0; i < 2u; ++i) {
        const uint32_t b = w.gw + i * w.nw;
        if (b >= batches) break;
        const uint32_t s = (w.it + i) & 1u;
        issue_batch<F, R>(p, b, w.stages + s * w.stage_bytes, &w.bars[s], G, lane);
    }
}

// This warp's batches of product p (its first two already in flight), x
// staged range-major at xs. The arithmetic of decode_kernel (matmul_decode.cu).
template <typename F, int R>
__device__ bool run_product(const MatmulArgs& p, const float* xs, Warp& w, uint32_t lane) {
    const uint32_t G = p.columns / 32u;
    const uint32_t lane_stride = x_lane_stride(G);
    const uint32_t batches = batch_count<R>(p);
    const bool gated = p.epilogue == kGated;
    const uint32_t lo = range_lo(lane, G), hi = range_lo(lane + 1u, G);
    const float4* xl = reinterpret_cast<const float4*>(xs + lane * lane_stride);
    uint32_t rb[F::kStreams], sl[F::kStreams], reg[F::kStreams];
#pragma unroll
    for (int q = 0; q < F::kStreams; ++q) {
        rb[q] = RowStreams<F>::row_bytes(q, G);
        sl[q] = RowStreams<F>::slot(q, G);
        reg[q] = q == 0 ? 0u : reg[q - 1] + R * sl[q - 1];
    }
    bool ok = true;
    uint32_t i = 0;
    for (uint32_t b = w.gw; b < batches; b += w.nw, ++i) {
        const uint32_t use = w.it + i, s = use & 1u;
        uint8_t* stage = w.stages + s * w.stage_bytes;
        if (!mbar_wait(&w.bars[s], (use >> 1) & 1u, p.fault)) {
            if (b + w.nw < batches) mbar_wait(&w.bars[s ^ 1u], ((use + 1u) >> 1) & 1u, nullptr);
            ok = false;
            ++i;
            break;
        }
        const Batch bt = locate_batch<R>(p, b);
        const uint8_t* seg[2][F::kStreams];
        {
            const MemberArgs& m0 = gated ? p.member[0] : p.member[bt.member];
#pragma unroll
            for (int q = 0; q < F::kStreams; ++q) {
                const uint64_t off = RowStreams<F>::base(q, m0.blocks) + static_cast<uint64_t>(m0.first_row + bt.local) * rb[q];
                seg[0][q] = stage + reg[q] + static_cast<uint32_t>(off & 15ull);
            }
            if (gated) {
                const MemberArgs& m1 = p.member[1];
#pragma unroll
                for (int q = 0; q < F::kStreams; ++q) {
                    const uint64_t off =
                        RowStreams<F>::base(q, m1.blocks) + static_cast<uint64_t>(m1.first_row + bt.local) * rb[q];
                    seg[1][q] = stage + reg[q] + (R > 1 ? R / 2 : 0) * sl[q] + static_cast<uint32_t>(off & 15ull);
                }
            }
        }
        if constexpr (R == 1) {
            float acc = 0.0f;
            for (uint32_t g = lo; g < hi; ++g) {
                F A;
                A.load(seg[0], g);
                chain_group1<F>(A, xl + (g - lo) * 8u, acc, std::make_integer_sequence<int, 32>{});
            }
            w.red[lane] = acc;
        } else {
            // R = 2: rows (0, 1) of the segment, or a gated output's gate and up rows.
            const bool la = bt.live > 0;
            const bool lb = gated ? la : bt.live > 1;
            const uint8_t* pa[F::kStreams];
            const uint8_t* pb[F::kStreams];
#pragma unroll
            for (int q = 0; q < F::kStreams; ++q) {
                pa[q] = seg[0][q];
                pb[q] = gated ? seg[1][q] : pa[q] + rb[q];
            }
            float aa = 0.0f, ab = 0.0f;
            for (uint32_t g = lo; g < hi; ++g) {
                F A, B;
                if (la) A.load(pa, g); else A.zero();
                if (lb) B.load(pb, g); else B.zero();
                chain_group<F>(A, B, xl + (g - lo) * 8u, aa, ab, std::make_integer_sequence<int, 32>{});
            }
            w.red[lane] = aa;
            w.red[kRedStride + lane] = ab;
        }
        fence_proxy_async();
        __syncwarp();
        if (b + 2u * w.nw < batches) issue_batch<F, R>(p, b + 2u * w.nw, stage, &w.bars[s], G, lane);
        float total = 0.0f;
        if (lane < static_cast<uint32_t>(R)) {
            const float4* rs = reinterpret_cast<const float4*>(w.red + lane * kRedStride);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float4 v = rs[q];
                total = total + v.x;
                total = total + v.y;
                total = total + v.z;
                total = total + v.w;
            }
        }
        if (gated) {
            const float up = __shfl_down_sync(0xFFFFFFFFu, total, R > 1 ? R / 2 : 1);
            if (lane < bt.live) {
                const uint32_t o = p.member[0].out_offset + bt.local + lane;
                p.out[0][o] = activate(p.activation, total) * up;
            }
        } else if (lane < bt.live) {
            const MemberArgs& m = p.member[bt.member];
            const uint32_t o = m.out_offset + bt.local + lane;
            if (p.epilogue == kQKV) p.out[bt.member][o] = total;
            else p.out[0][o] = total;
        }
        __syncwarp();
    }
    w.it += i;
    return ok;
}

// A gated product always takes batches of two rows (an output's gate row
// and up row share a batch).
template <int R>
__device__ void prefetch_any(const MatmulArgs& p, Warp& w, uint32_t lane) {
    const bool gated = p.epilogue == kGated;
    switch (p.format) {
        case kQ4_0: gated ? prefetch_product<Q4_0, 2>(p, w, lane) : prefetch_product<Q4_0, R>(p, w, lane); break;
        case kQ8_0: gated ? prefetch_product<Q8_0, 2>(p, w, lane) : prefetch_product<Q8_0, R>(p, w, lane); break;
        default: gated ? prefetch_product<Q6_K, 2>(p, w, lane) : prefetch_product<Q6_K, R>(p, w, lane); break;
    }
}
template <int R>
__device__ bool run_any(const MatmulArgs& p, const float* xs, Warp& w, uint32_t lane) {
    const bool gated = p.epilogue == kGated;
    switch (p.format) {
        case kQ4_0: return gated ? run_product<Q4_0, 2>(p, xs, w, lane) : run_product<Q4_0, R>(p, xs, w, lane);
        case kQ8_0: return gated ? run_product<Q8_0, 2>(p, xs, w, lane) : run_product<Q8_0, R>(p, xs, w, lane);
        default: return gated ? run_product<Q6_K, 2>(p, xs, w, lane) : run_product<Q6_K, R>(p, xs, w, lane);
    }
}

// x[0..K) from global memory into the range-major stage (every warp copies
// part of every range, as decode_kernel does).
__device__ void stage_x(const float* x, uint32_t K, float* xs, uint32_t warps) {
    const uint32_t G = K / 32u, lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t lane_stride = x_lane_stride(G);
    const uint32_t lo = range_lo(lane, G), hi = range_lo(lane + 1u, G);
    const float4* xg = reinterpret_cast<const float4*>(x);
    float4* dst = reinterpret_cast<float4*>(xs + lane * lane_stride);
    for (uint32_t g = lo + warp; g < hi; g += warps)
#pragma unroll
        for (int v = 0; v < 8; ++v) dst[(g - lo) * 8u + v] = __ldcg(xg + g * 8u + v);
}

// The reference's 256-way halving tree (norm.wgsl:67-78), threads 0..255
// holding the partials; every thread of the CTA takes part in the barriers.
__device__ float tree_sum256(float v, float* scratch) {
    const int i = threadIdx.x;
    if (i < 256) scratch[i] = v;
    __syncthreads();
#pragma unroll
    for (int stride = 128; stride >= 32; stride >>= 1) {
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
    __syncthreads();
    return total;
}

// norm_kernel's arithmetic for one row (norm.cu): with `add`, x = hidden +
// y (y post-normed first when post_gain), written to hidden_out when given;
// then normed = (x·r)·g — into the range-major x stage (xs) when xs is
// given, else into normed_out.
__device__ void norm_row(const float* hidden, const float* y, const float* post_gain, const float* gain,
                         float* hidden_out, uint32_t width, float epsilon, float* scratch, float* xs,
                         float* normed_out) {
    const uint32_t vec4s = width / 4u, t = threadIdx.x;
    const float n = static_cast<float>(width);
    float4 x[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t i = t + k * 256u;
        x[k] = (t < 256u && i < vec4s) ? __ldcg(reinterpret_cast<const float4*>(hidden) + i)
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (y) {
        float4 yy[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t i = t + k * 256u;
            yy[k] = (t < 256u && i < vec4s) ? __ldcg(reinterpret_cast<const float4*>(y) + i)
                                             : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        if (post_gain) {
            float squares = 0.0f;
#pragma unroll
            for (int k = 0; k < 4; ++k)
                if (t < 256u && t + k * 256u < vec4s) squares = squares + dot4(yy[k], yy[k]);
            const float r = 1.0f / sqrtf(tree_sum256(squares, scratch) / n + epsilon);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t i = t + k * 256u;
                if (t < 256u && i < vec4s) {
                    const float4 g = reinterpret_cast<const float4*>(post_gain)[i];
                    yy[k] = make_float4(((yy[k].x * r) * g.x) * 1.0f, ((yy[k].y * r) * g.y) * 1.0f,
                                        ((yy[k].z * r) * g.z) * 1.0f, ((yy[k].w * r) * g.w) * 1.0f);
                }
            }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t i = t + k * 256u;
            if (t < 256u && i < vec4s) {
                x[k] = make_float4(x[k].x + yy[k].x, x[k].y + yy[k].y, x[k].z + yy[k].z, x[k].w + yy[k].w);
                if (hidden_out) reinterpret_cast<float4*>(hidden_out)[i] = x[k];
            }
        }
    }
    float squares = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; ++k)
        if (t < 256u && t + k * 256u < vec4s) squares = squares + dot4(x[k], x[k]);
    const float r = 1.0f / sqrtf(tree_sum256(squares, scratch) / n + epsilon);
    const uint32_t G = width / 32u, lane_stride = x_lane_stride(G);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t i = t + k * 256u;
        if (t < 256u && i < vec4s) {
            const float4 g = reinterpret_cast<const float4*>(gain)[i];
            const float4 v = make_float4((x[k].x * r) * g.x, (x[k].y * r) * g.y, (x[k].z * r) * g.z, (x[k].w * r) * g.w);
            if (xs) {
                const uint32_t e = 4u * i, grp = e / 32u, lr = lane_of(grp, G);
                *reinterpret_cast<float4*>(xs + lr * lane_stride + (grp - range_lo(lr, G)) * 32u + e % 32u) = v;
            } else {
                reinterpret_cast<float4*>(normed_out)[i] = v;
            }
        }
    }
}

__device__ __forceinline__ void store_f16x4(uint16_t* dst, float4 v) {
    const uint32_t lo = static_cast<uint32_t>(f32_to_f16_sat(v.x)) | (static_cast<uint32_t>(f32_to_f16_sat(v.y)) << 16);
    const uint32_t hi = static_cast<uint32_t>(f32_to_f16_sat(v.z)) | (static_cast<uint32_t>(f32_to_f16_sat(v.w)) << 16);
    *reinterpret_cast<uint2*>(dst) = make_uint2(lo, hi);
}

// rope_kernel's arithmetic (rope.cu) for kv head `h`'s G query heads — into
// qs, scaled into log2 units as the attention stage stages them — and, with
// `kv`, its key and value heads into the cache slot of position p. Threads
// [0, heads·lanes) rounded up to a warp take part (the head tree's shuffles
// are warp-wide); cosines and sines hold the position's d/2 angles.
__device__ void rope_heads(const FusedArgs& a, const FusedLayer& L, uint32_t h, uint32_t p, bool kv, float* qs,
                           const float* cosines, const float* sines) {
    const uint32_t d = a.d, lanes = d / 8u, G = a.Hq / a.Hkv;
    const uint32_t heads = G + (kv ? 2u : 0u);
    const uint32_t span = (heads * lanes + 31u) / 32u * 32u;
    const uint32_t t = threadIdx.x;
    if (t >= span) return;
    const uint32_t head = t / lanes, lane = t % lanes;
    const bool real = head < heads;
    const bool is_query = head < G;
    const bool is_value = kv && head == G + 1u;
    float4 x0 = make_float4(0.f, 0.f, 0.f, 0.f), x1 = x0;
    if (real) {
        const float* src = is_query ? a.q + (static_cast<size_t>(h) * G + head) * d
                                    : (is_value ? a.v : a.k) + static_cast<size_t>(h) * d;
        x0 = __ldcg(reinterpret_cast<const float4*>(src) + lane);
        x1 = __ldcg(reinterpret_cast<const float4*>(src) + lane + lanes);
    }
    float r = 1.0f;
    if (L.q_norm) {
        float v = dot4(x0, x0) + dot4(x1, x1);
        for (uint32_t stride = lanes / 2u; stride > 0; stride >>= 1)
            v = v + __shfl_down_sync(0xFFFFFFFFu, v, stride, lanes);
        const float total = __shfl_sync(0xFFFFFFFFu, v, 0, lanes);
        r = 1.0f / sqrtf(total / static_cast<float>(d) + a.epsilon);
    }
    if (!real) return;
    if (!is_value) {
        const float* gain = is_query ? L.q_norm : L.k_norm;
        if (gain) {
            const float4 g0 = reinterpret_cast<const float4*>(gain)[lane];
            const float4 g1 = reinterpret_cast<const float4*>(gain)[lane + lanes];
            x0 = make_float4((x0.x * r) * g0.x, (x0.y * r) * g0.y, (x0.z * r) * g0.z, (x0.w * r) * g0.w);
            x1 = make_float4((x1.x * r) * g1.x, (x1.y * r) * g1.y, (x1.z * r) * g1.z, (x1.w * r) * g1.w);
        }
        if (a.halves) {
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
            float* e[2] = {&x0.x, &x1.x};
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const uint32_t k = (hh ? d / 4u : 0u) + 2u * lane + c;
                    const float u = e[hh][2 * c], w = e[hh][2 * c + 1];
                    e[hh][2 * c] = fmaf(u, cosines[k], (-w) * sines[k]);
                    e[hh][2 * c + 1] = fmaf(w, cosines[k], u * sines[k]);
                }
            }
        }
    }
    if (is_query) {
        float4* dst = reinterpret_cast<float4*>(qs + head * d);
        const float sc = a.scale_log2e;
        dst[lane] = make_float4(x0.x * sc, x0.y * sc, x0.z * sc, x0.w * sc);
        dst[lane + lanes] = make_float4(x1.x * sc, x1.y * sc, x1.z * sc, x1.w * sc);
    } else {
        uint16_t* cache = is_value ? L.value_cache : L.key_cache;
        uint16_t* dst = cache + (static_cast<size_t>(p % L.slots) * a.Hkv + h) * d;
        store_f16x4(dst + 4u * lane, x0);
        store_f16x4(dst + 4u * (lane + lanes), x1);
    }
}

// One (kv head, chunk) item of the attention stage: attention_kernel's
// arithmetic (attention.cu) for a single row at position p, its G queries.
__device__ void attention_item(const FusedArgs& a, const FusedLayer& L, uint32_t h, uint32_t c, uint32_t p,
                               uint8_t* area) {
    const uint32_t d = a.d, G = a.Hq / a.Hkv, B = 2048u / d, tiles = kChunkF / B;
    const uint32_t nt = blockDim.x, lane = threadIdx.x & 31u, wid = threadIdx.x >> 5;
    uint16_t* ks = reinterpret_cast<uint16_t*>(area);
    uint16_t* vs = ks + kChunkF * d;
    float* qs = reinterpret_cast<float*>(vs + kChunkF * d);   // [G][d]
    float* ps = qs + 16u * d;                                  // [G][64]
    float* alpha = ps + 16u * kChunkF;                          // [G][8]
    float* stat = alpha + 16u * 8u;                             // [G][4]
    float* cosines = stat + 16u * 4u;                           // [d/2]
    float* sines = cosines + 128u;                              // [d/2]
    const uint32_t key0 = c * kChunkF;
    const bool last_chunk = c == p / kChunkF;
    // the position's angles (rope_kernel)
    for (uint32_t k = threadIdx.x; k < d / 2u; k += nt) {
        float t = static_cast<float>(p) * L.turns[k];
        if (a.factors) t = t / a.factors[k];
        const float angle = 6.283185307179586f * (t - rintf(t));
        sincos_turn(angle, &sines[k], &cosines[k]);
    }
    __syncthreads();
    rope_heads(a, L, h, p, last_chunk, qs, cosines, sines);
    __syncthreads();   // the new key and value are in the cache (global), visible to the CTA
    // keys key0 .. min(key0 + 64, p + 1)
    const uint32_t j_hi = min(key0 + kChunkF, p + 1u);
    const uint32_t words = d / 8u;
    for (uint32_t i = threadIdx.x; i < (j_hi - key0) * words; i += nt) {
        const uint32_t b = i / words, w = i % words;
        const size_t at = (static_cast<size_t>((key0 + b) % L.slots) * a.Hkv + h) * d;
        reinterpret_cast<uint4*>(ks + b * d)[w] = reinterpret_cast<const uint4*>(L.key_cache + at)[w];
        reinterpret_cast<uint4*>(vs + b * d)[w] = reinterpret_cast<const uint4*>(L.value_cache + at)[w];
    }
    __syncthreads();
    const uint32_t early = earliest_f(p, L.window);
    for (uint32_t i = threadIdx.x; i < G * kChunkF; i += nt) {
        const uint32_t m = i / kChunkF, b = i % kChunkF;
        const uint32_t j = key0 + b;
        float s = 0.0f;
        if (j <= p && j >= early) {
            const float4* q4 = reinterpret_cast<const float4*>(qs + m * d);
            const uint2* k4 = reinterpret_cast<const uint2*>(ks + b * d);
#pragma unroll 8
            for (uint32_t w = 0; w < d / 4u; ++w) {
                const uint2 kw = k4[w];
                const float4 kk = make_float4(fp16_bits_to_f32(kw.x & 0xFFFF), fp16_bits_to_f32(kw.x >> 16),
                                              fp16_bits_to_f32(kw.y & 0xFFFF), fp16_bits_to_f32(kw.y >> 16));
                s = s + dot4(q4[w], kk);
            }
        }
        ps[m * kChunkF + b] = s;
    }
    __syncthreads();
    for (uint32_t m = wid; m < G; m += nt / 32u) {
        bool chunk_live = false;
        float chunk_m = 0.0f, chunk_l = 0.0f;
        for (uint32_t t = 0; t < tiles; ++t) {
            const uint32_t b = t * B + lane;
            const uint32_t j = key0 + b;
            const bool live = lane < B && j <= p && j >= early;
            const float s = live ? ps[m * kChunkF + b] : 0.0f;
            float top_tile = live ? s : -INFINITY;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) top_tile = fmaxf(top_tile, __shfl_xor_sync(0xFFFFFFFFu, top_tile, o));
            const bool seen = __any_sync(0xFFFFFFFFu, live);
            float al = 1.0f;
            if (seen) {
                const float old = chunk_live ? chunk_m : top_tile;
                chunk_live = true;
                const float top = fmaxf(old, top_tile);
                al = old == top ? 1.0f : exp2_np(old - top);
                const float e = live ? exp2_np(s - top) : 0.0f;
                if (lane < B) ps[m * kChunkF + b] = e;
                float sum = 0.0f;
                for (uint32_t i = 0; i < B; ++i) sum = sum + __shfl_sync(0xFFFFFFFFu, e, i);
                chunk_l = fmaf(chunk_l, al, sum);
                chunk_m = top;
            } else if (lane < B) {
                ps[m * kChunkF + b] = 0.0f;
            }
            if (lane == 0) alpha[m * 8u + t] = al;
        }
        if (lane == 0) {
            stat[m * 4u + 0] = chunk_m;
            stat[m * 4u + 1] = chunk_live ? chunk_l : 0.0f;
        }
    }
    __syncthreads();
    const uint32_t valid = min(kChunkF, p + 1u - key0);
    for (uint32_t i = threadIdx.x; i < G * d; i += nt) {
        const uint32_t m = i / d, e = i % d;
        float o = 0.0f;
        for (uint32_t t = 0; t < tiles; ++t) {
            o = o * alpha[m * 8u + t];
            const uint32_t b_end = min((t + 1u) * B, valid);
#pragma unroll 8
            for (uint32_t b = t * B; b < b_end; ++b) o = fmaf(ps[m * kChunkF + b], fp16_bits_to_f32(vs[b * d + e]), o);
        }
        const size_t at = static_cast<size_t>(c) * a.Hq + h * G + m;
        a.partials[at * d + e] = o;
        if (e == 0) {
            a.stats[at * 2u] = stat[m * 4u];
            a.stats[at * 2u + 1u] = stat[m * 4u + 1u];
        }
    }
    __syncthreads();
}

// The fold of attention_kernel (attention.cu) for (query head hq, dimension
// e) at position p: the live chunks' states in chunk order, then O / l.
__device__ void fold_one(const FusedArgs& a, const FusedLayer& L, uint32_t hq, uint32_t e, uint32_t p) {
    const uint32_t d = a.d;
    const uint32_t c0 = earliest_f(p, L.window) / kChunkF, c1 = p / kChunkF;
    bool live = false;
    float run_m = 0.0f, run_l = 0.0f, o = 0.0f;
    for (uint32_t cc = c0; cc <= c1; cc += 8u) {
        float co[8], cm[8], cl[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const size_t at = static_cast<size_t>(cc + k) * a.Hq + hq;
            const bool in = cc + k <= c1;
            co[k] = in ? __ldcg(a.partials + at * d + e) : 0.0f;
            cm[k] = in ? __ldcg(a.stats + at * 2u) : 0.0f;
            cl[k] = in ? __ldcg(a.stats + at * 2u + 1u) : 0.0f;
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            if (cc + k > c1) break;
            float fa, fb, fm;
            if (!live) { fa = 0.0f; fb = 1.0f; fm = cm[k]; }
            else if (run_m == cm[k]) { fa = 1.0f; fb = 1.0f; fm = run_m; }
            else if (run_m > cm[k]) { fa = 1.0f; fb = exp2_np(cm[k] - run_m); fm = run_m; }
            else { fa = exp2_np(run_m - cm[k]); fb = 1.0f; fm = cm[k]; }
            run_l = fmaf(run_l, fa, cl[k] * fb);
            o = fmaf(o, fa, co[k] * fb);
            run_m = fm;
            live = true;
        }
    }
    a.att[static_cast<size_t>(hq) * d + e] = live ? o / run_l : 0.0f;
}

// gather_kernel's arithmetic (gather.cu) for group g of the token's row.
template <typename F, int k>
__device__ __forceinline__ void gather_put(const F& f, const typename F::Consts& c, float scale, float* out) {
    out[k] = F::template weight<k>(f, c) * scale;
}
template <typename F, int... ks>
__device__ __forceinline__ void gather_all(const F& f, float scale, float* out, std::integer_sequence<int, ks...>) {
    const typename F::Consts c = f.consts();
    (gather_put<F, ks>(f, c, scale, out), ...);
}
template <typename F>
__device__ void gather_group(const FusedArgs& a, uint32_t token, uint32_t g, float* hidden) {
    const uint32_t groups = a.H / 32u;
    const uint8_t* s[F::kStreams];
#pragma unroll
    for (int q = 0; q < F::kStreams; ++q)
        s[q] = a.embed_piece + RowStreams<F>::base(q, a.embed_blocks) +
               static_cast<uint64_t>(token) * RowStreams<F>::row_bytes(q, groups);
    F f;
    f.load(s, g);
    float w[32];
    gather_all<F>(f, a.embed_scale, w, std::make_integer_sequence<int, 32>{});
    float4* out = reinterpret_cast<float4*>(hidden + g * 32u);
#pragma unroll
    for (int v = 0; v < 8; ++v) out[v] = make_float4(w[4 * v], w[4 * v + 1], w[4 * v + 2], w[4 * v + 3]);
}

template <int R>
__global__ void __launch_bounds__(512, 1) fused_step_kernel(const FusedArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t warps = blockDim.x / 32u, warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t n = gridDim.x;
    // shared memory: x stage | norm scratch | per warp (bars, red, 2 slots) | attention area
    float* xs = reinterpret_cast<float*>(smem);
    float* scratch = xs + a.x_stage_floats;
    uint8_t* wbase = reinterpret_cast<uint8_t*>(scratch + 256);
    const uint32_t warp_bytes = 16u + 2u * kRedStride * 4u + 2u * a.stage_bytes;   // range sums of up to 2 rows
    uint8_t* mine = wbase + warp * warp_bytes;
    uint8_t* area = wbase + warps * warp_bytes;
    Warp w;
    w.bars = reinterpret_cast<uint64_t*>(mine);
    w.red = reinterpret_cast<float*>(mine + 16);
    w.stages = mine + 16u + 2u * kRedStride * 4u;
    w.stage_bytes = a.stage_bytes;
    w.it = 0;
    w.gw = blockIdx.x * warps + warp;
    w.nw = n * warps;
    if (lane == 0) {
        mbar_init(&w.bars[0], 1);
        mbar_init(&w.bars[1], 1);
        fence_barrier_init();
    }
    __syncwarp();

    const uint32_t p = *a.state;
    const uint32_t token = a.fed ? a.sampled[0] : a.ids[0];
    bool ok = true;
    // the first layer's QKV weights in flight while the token is gathered
    prefetch_any<R>(a.layers[0].qkv, w, lane);
    {
        const uint32_t groups = a.H / 32u;
        for (uint32_t g = blockIdx.x * blockDim.x + threadIdx.x; g < groups; g += n * blockDim.x) {
            switch (a.embed_format) {
                case kQ4_0: gather_group<Q4_0>(a, token, g, a.hidden[0]); break;
                case kQ8_0: gather_group<Q8_0>(a, token, g, a.hidden[0]); break;
                default: gather_group<Q6_K>(a, token, g, a.hidden[0]); break;
            }
        }
    }
    ok = grid_barrier(a.bar, n, a.fault);
    uint32_t cur = 0;
    const float* pending_post = nullptr;
    bool pending_add = false;
    for (uint32_t l = 0; l < a.n_layers && ok; ++l) {
        const FusedLayer& L = a.layers[l];
        // A: attention norm, QKV
        norm_row(a.hidden[cur], pending_add ? a.out : nullptr, pending_post, L.attn_norm,
                 (pending_add && blockIdx.x == 0) ? a.hidden[cur ^ 1u] : nullptr, a.H, a.epsilon, scratch, xs, nullptr);
        if (pending_add) cur ^= 1u;
        __syncthreads();
        ok = __syncthreads_and(run_any<R>(L.qkv, xs, w, lane));
        if (!(ok = grid_barrier(a.bar, n, a.fault) && ok)) break;
        // B: rope and the chunks' states
        {
            const uint32_t c_lo = earliest_f(p, L.window) / kChunkF, chunks = p / kChunkF - c_lo + 1u;
            for (uint32_t item = blockIdx.x; item < a.Hkv * chunks; item += n)
                attention_item(a, L, item % a.Hkv, c_lo + item / a.Hkv, p, area);
        }
        prefetch_any<R>(L.o, w, lane);
        if (!(ok = grid_barrier(a.bar, n, a.fault))) break;
        // C: the fold
        for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < a.Hq * a.d; i += n * blockDim.x)
            fold_one(a, L, i / a.d, i % a.d, p);
        if (!(ok = grid_barrier(a.bar, n, a.fault))) break;
        // D: O
        stage_x(a.att, a.Hq * a.d, xs, warps);
        __syncthreads();
        ok = __syncthreads_and(run_any<R>(L.o, xs, w, lane));
        prefetch_any<R>(L.gate_up, w, lane);
        if (!(ok = grid_barrier(a.bar, n, a.fault) && ok)) break;
        // E: feed-forward norm with the add, gate|up
        norm_row(a.hidden[cur], a.out, L.post_attn_norm, L.ffn_norm, blockIdx.x == 0 ? a.hidden[cur ^ 1u] : nullptr,
                 a.H, a.epsilon, scratch, xs, nullptr);
        cur ^= 1u;
        __syncthreads();
        ok = __syncthreads_and(run_any<R>(L.gate_up, xs, w, lane));
        prefetch_any<R>(L.down, w, lane);
        if (!(ok = grid_barrier(a.bar, n, a.fault) && ok)) break;
        // F: down
        stage_x(a.act, a.ffn, xs, warps);
        __syncthreads();
        ok = __syncthreads_and(run_any<R>(L.down, xs, w, lane));
        if (l + 1u < a.n_layers) prefetch_any<R>(a.layers[l + 1u].qkv, w, lane);
        if (!(ok = grid_barrier(a.bar, n, a.fault) && ok)) break;
        pending_add = true;
        pending_post = L.post_ffn_norm;
    }
    if (ok) {
        // the final norm of the last (only) token, for the head
        if (blockIdx.x == 0)
            norm_row(a.hidden[cur], a.out, pending_post, a.output_norm, nullptr, a.H, a.epsilon, scratch, nullptr,
                     a.normed);
    } else {
        // leave no bulk copy writing this CTA's shared memory: the slots of
        // batches in flight (at most two) land or run out, bounded
        mbar_wait(&w.bars[w.it & 1u], (w.it >> 1) & 1u, nullptr);
        mbar_wait(&w.bars[(w.it + 1u) & 1u], ((w.it + 1u) >> 1) & 1u, nullptr);
    }
}

}  // namespace

FusedPlan fused_plan(uint32_t max_columns, uint32_t max_row_stage, uint32_t gated_row_stage, uint32_t head_dim,
                     int sm_count, int dev) {
    FusedPlan plan{};
    const uint32_t Gmax = max_columns / 32u;
    const size_t x_stage = static_cast<size_t>(32u) * x_lane_stride(Gmax) * 4u;
    const size_t attn = static_cast<size_t>(2u) * kChunkF * head_dim * 2u + (16u * head_dim + 16u * kChunkF + 16u * 8u +
                                                                              16u * 4u + 256u) * 4u;
    int max_smem = 0;
    cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    const int configs[4][2] = {{16, 2}, {16, 1}, {8, 2}, {8, 1}};
    for (const auto& c : configs) {
        const uint32_t W = c[0], R = c[1];
        const uint32_t stage_bytes = R * max_row_stage > 2u * gated_row_stage ? R * max_row_stage : 2u * gated_row_stage;
        const size_t smem = x_stage + 256u * 4u + W * (16u + 2u * kRedStride * 4u + 2ull * stage_bytes) + attn;
        if (smem + 1024u <= static_cast<size_t>(max_smem)) {
            plan.warps = W;
            plan.R = R;
            plan.stage_bytes = stage_bytes;
            plan.x_stage_floats = static_cast<uint32_t>(x_stage / 4u);
            plan.smem = smem;
            plan.ctas = static_cast<uint32_t>(sm_count);
            return plan;
        }
    }
    return plan;   // warps == 0: does not fit
}

cudaError_t fused_step_run(const FusedArgs& a, const FusedPlan& plan, cudaStream_t stream) {
    auto kernel = plan.R == 2 ? fused_step_kernel<2> : fused_step_kernel<1>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(plan.smem));
    if (e != cudaSuccess) return e;
    int blocks = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, plan.warps * 32, plan.smem);
    if (e != cudaSuccess) return e;
    if (blocks < 1) return cudaErrorCooperativeLaunchTooLarge;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(plan.ctas);
    cfg.blockDim = dim3(plan.warps * 32u);
    cfg.dynamicSmemBytes = plan.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, a);
}

}  // namespace cb
