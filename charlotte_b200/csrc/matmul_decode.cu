// Decode matrix products: y = W·x for one token (or each of a few tokens),
// W in GGUF Q4_0, Q8_0 or repacked Q6_K read from the reference's device
// layout and decoded in the load path (plainsight-systems/charlotte,
// src/core/kernels/matmul/matmul.wgsl decode_write/decode_qkv/decode_gated/
// decode_gated_input, :287-361).
//
// Order of addition — the reference's, fixed by K alone (matmul.h:34-50):
// a row's G = K/32 groups are cut into 32 ranges at floor(r·G/32); lane r of
// a warp sums range r of each of its rows as one fma chain from zero, k in
// order; the 32 range sums meet in shared memory and one lane adds them to a
// total from zero, r in order. So every output is bit-identical to the CPU
// oracle's and to the reference's prefill form of the same token.
//
// B200 mapping.
//  - A warp owns batches of R rows. Small products (most of a decode step)
//    take the latency shape: R from 2 and W warps a CTA chosen so that every
//    warp has one batch and the grid is at most one CTA an SM — all copies
//    are issued before the wait on the launch before, every CTA is resident
//    beside that launch's (none starts late, after it has exited), and x is
//    read once an SM. Larger products stream: several batches a warp through
//    a two-stage ring, the copy of batch i+2 in flight while batch i is
//    worked.
//  - Each batch's row streams (codes, scales, ...) are brought into the
//    warp's shared memory by bulk asynchronous copies (cp.async.bulk, the
//    untiled TMA), completing on an mbarrier.
//  - The first two batches' copies are issued before griddepcontrol.wait:
//    weights are never written on the device, so under programmatic
//    dependent launch a product's weight stream overlaps the launch before it;
//    only x, the previous launch's output, waits.
//  - Rows are worked two at a time: one paired fma (fma.rn.f32x2, two fmas
//    each rounded once) decodes a weight of each row exactly (formats.cuh),
//    one accumulates both, with x held doubled ((x_k, x_k)) in shared memory
//    as the pair's operand. In batches of four or more rows the pairs'
//    chains advance together, k outermost: one read of x serves every pair
//    (chain_group_rows).
//  - Batches never straddle members, so a batch's rows come in one bulk copy
//    per stream (two for a gated batch: its gate rows and its up rows).
//  - x is staged once per CTA in shared memory range-major, a 16-byte skew
//    per range, so the lanes' 128-bit reads fall in distinct banks; the row
//    is read from global memory in order (each warp one contiguous span).
//  - Every mbarrier wait is bounded (tma.cuh): a copy that never lands sets
//    the launch's fault word, which the host reports as a failed step.
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>
#include <utility>

#include "formats.cuh"
#include "matmul.h"
#include "numerics.cuh"
#include "gemv_common.cuh"
#include "tma.cuh"

namespace cb {

namespace {

constexpr int kWarps = 4;
constexpr int kMaxDecodeSmem = 220 * 1024;

// The reference's 256-way halving tree (norm.wgsl:67-78) on the first 128
// threads of a CTA (the rest only meet its barriers): thread t holds partials
// t and t+128 (the tree's first level adds exactly those two), then the
// levels 64 and 32 in shared memory and the shuffles of the last warp, as
// norm_kernel does.
__device__ __forceinline__ float tree_sum_pairs(float lo, float hi, float* scratch) {
    const uint32_t t = threadIdx.x;
    if (t < 128u) scratch[t] = lo + hi;
    __syncthreads();
    if (t < 64u) scratch[t] = scratch[t] + scratch[t + 64u];
    __syncthreads();
    if (t < 32u) scratch[t] = scratch[t] + scratch[t + 32u];
    __syncthreads();
    if (t < 32u) {
        float w = scratch[t];
#pragma unroll
        for (int stride = 16; stride > 0; stride >>= 1) w = w + __shfl_down_sync(0xFFFFFFFFu, w, stride);
        if (t == 0) scratch[0] = w;
    }
    __syncthreads();
    const float total = scratch[0];
    __syncthreads();
    return total;
}

// norm_kernel's row (norm.cu) for one token on the first 128 threads of a
// CTA: thread t does the work of norm_kernel's threads t and t+128 (vec4s
// t + 128h + 256k), the same operations in the same order. The hidden row
// and y come by asynchronous copies, each thread's own elements, into the x
// stage's space (twice the row: room for both), so no registers wait on the
// loads; the normed row then goes to the x stage, range-major with every
// float doubled, once every thread holds its own normed elements; CTA 0
// writes the add. Threads from 128 up hold no elements and only meet the
// barriers.
__device__ __forceinline__ void norm_row128(const MatmulArgs& a, float* xs, uint32_t G, uint32_t lane_stride) {
    __shared__ float scratch[128];
    const uint32_t width = a.columns, t = threadIdx.x;
    const uint32_t vec4s = t < 128u ? width / 4u : 0u;
    const float n = static_cast<float>(width);
    float4* th = reinterpret_cast<float4*>(xs);
    float4* ty = th + width / 4u;
    const float4* hg = reinterpret_cast<const float4*>(a.norm_hidden);
    const float4* yg = reinterpret_cast<const float4*>(a.norm_y);
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t i = t + 128u * h + 256u * k;
            if (i < vec4s) {
                cp_async16(th + i, hg + i);
                if (yg) cp_async16(ty + i, yg + i);
            }
        }
    cp_async_wait_all();
    if (yg) {
        if (a.norm_post_gain) {
            float sq[2] = {0.0f, 0.0f};
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const uint32_t i = t + 128u * h + 256u * k;
                    if (i < vec4s) sq[h] = sq[h] + dot4(ty[i], ty[i]);
                }
            const float r = 1.0f / sqrtf(tree_sum_pairs(sq[0], sq[1], scratch) / n + a.norm_epsilon);
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const uint32_t i = t + 128u * h + 256u * k;
                    if (i < vec4s) {
                        const float4 g = reinterpret_cast<const float4*>(a.norm_post_gain)[i];
                        const float4 y = ty[i];
                        ty[i] = make_float4(((y.x * r) * g.x) * 1.0f, ((y.y * r) * g.y) * 1.0f,
                                            ((y.z * r) * g.z) * 1.0f, ((y.w * r) * g.w) * 1.0f);
                    }
                }
        }
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t i = t + 128u * h + 256u * k;
                if (i < vec4s) {
                    const float4 x = th[i], y = ty[i];
                    const float4 v = make_float4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w);
                    th[i] = v;
                    if (blockIdx.x == 0 && a.norm_hidden_out) reinterpret_cast<float4*>(a.norm_hidden_out)[i] = v;
                }
            }
    }
    float sq[2] = {0.0f, 0.0f};
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t i = t + 128u * h + 256u * k;
            if (i < vec4s) sq[h] = sq[h] + dot4(th[i], th[i]);
        }
    const float r = 1.0f / sqrtf(tree_sum_pairs(sq[0], sq[1], scratch) / n + a.norm_epsilon);
    // The normed elements into y's half (read by their own thread only, dead
    // after the add), then, every thread past the barrier, into registers
    // and the stage's doubled layout (which spans both halves).
    float4* tv = th + width / 4u;
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t i = t + 128u * h + 256u * k;
            if (i < vec4s) {
                const float4 g = reinterpret_cast<const float4*>(a.norm_gain)[i];
                const float4 x = th[i];
                tv[i] = make_float4((x.x * r) * g.x, (x.y * r) * g.y, (x.z * r) * g.z, (x.w * r) * g.w);
            }
        }
    float4 v[2][4];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t i = t + 128u * h + 256u * k;
            v[h][k] = i < vec4s ? tv[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    __syncthreads();   // every thread holds its elements: the stage may overwrite the rows
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t i = t + 128u * h + 256u * k;
            if (i < vec4s) {
                const uint32_t e = 4u * i, grp = e / 32u, lr = lane_of(grp, G);
                float4* d = reinterpret_cast<float4*>(xs + lr * lane_stride + (grp - range_lo(lr, G)) * 64u + 2u * (e % 32u));
                d[0] = make_float4(v[h][k].x, v[h][k].x, v[h][k].y, v[h][k].y);
                d[1] = make_float4(v[h][k].z, v[h][k].z, v[h][k].w, v[h][k].w);
            }
        }
}

// Whether a batch's row pairs run their chains together (chain_group_rows):
// batches of 4 or more rows of the formats whose decoded state stays in
// registers for every pair at once (Q4_1 and BF16 would spill).
template <typename F, int R>
constexpr bool kRowsTogether = R >= 4 && (std::is_same<F, Q4_0>::value || std::is_same<F, Q8_0>::value ||
                                          std::is_same<F, Q6_K>::value);

template <typename F, int R, int W>
__global__ void __launch_bounds__(W * 32) decode_kernel(const MatmulArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t G = a.columns / 32u;
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t lane_stride = x2_lane_stride(G);
    const uint32_t stage_bytes = RowStreams<F>::row_stage(G) * R;
    const uint32_t batches = batch_count<R>(a);
    const uint32_t stride = gridDim.x * W;
    const bool gated = a.epilogue == kGated;
    const uint32_t spin = spin_limit_of(a.fault);   // read early: off the first wait's path

    // Shared memory: x (range-major, each float doubled), then per warp: 2
    // barriers, range sums, 2 stages.
    float* xs = reinterpret_cast<float*>(smem);
    const uint32_t x_bytes = 32u * lane_stride * 4u;
    const uint32_t warp_bytes = 16u + R * kRedStride * 4u + 2u * stage_bytes;
    uint8_t* wbase = smem + x_bytes + warp * warp_bytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(wbase);
    float* red = reinterpret_cast<float*>(wbase + 16);
    uint8_t* stages = wbase + 16u + R * kRedStride * 4u;

    if (lane == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        fence_barrier_init();
    }
    __syncwarp();
    const uint32_t first = blockIdx.x * W + warp;
    if (first < batches) issue_batch<F, R>(a, first, stages, &bars[0], G, lane);
    if (first + stride < batches) issue_batch<F, R>(a, first + stride, stages + stage_bytes, &bars[1], G, lane);

    grid_dependency_wait();

    // x, range-major: lane r's groups at r·lane_stride (64 floats a group,
    // each float doubled), a 16-byte skew a range. The row's 16-byte chunks
    // are dealt to all threads in row order (each warp reads one contiguous
    // span). Or, with the norm folded in, the normed row computed here.
    const uint32_t t = blockIdx.y;
    const uint32_t lo = range_lo(lane, G), hi = range_lo(lane + 1u, G);
    if (a.norm_gain) {
        norm_row128(a, xs, G, lane_stride);
    } else {
        const float4* xg = reinterpret_cast<const float4*>(a.x + static_cast<size_t>(t) * a.x_stride);
#pragma unroll 2
        for (uint32_t c = threadIdx.x; c < G * 8u; c += W * 32u) {
            const float4 v = __ldcg(xg + c);
            const uint32_t grp = c / 8u, lr = lane_of(grp, G);
            float4* d = reinterpret_cast<float4*>(xs + lr * lane_stride + (grp - range_lo(lr, G)) * 64u + (c % 8u) * 8u);
            d[0] = make_float4(v.x, v.x, v.y, v.y);
            d[1] = make_float4(v.z, v.z, v.w, v.w);
        }
    }
    __syncthreads();
    grid_dependents_launch();
    const float4* xl = reinterpret_cast<const float4*>(xs + lane * lane_stride);

    // Per stream: a row's bytes, a slot's bytes, the region's offset in a stage.
    uint32_t rb[F::kStreams], sl[F::kStreams], reg[F::kStreams];
#pragma unroll
    for (int q = 0; q < F::kStreams; ++q) {
        rb[q] = RowStreams<F>::row_bytes(q, G);
        sl[q] = RowStreams<F>::slot(q, G);
        reg[q] = q == 0 ? 0u : reg[q - 1] + R * sl[q - 1];
    }

    uint32_t i = 0;
    for (uint32_t b = first; b < batches; b += stride, ++i) {
        const uint32_t s = i & 1u;
        uint8_t* stage = stages + s * stage_bytes;
        if (!mbar_wait(&bars[s], (i >> 1) & 1u, a.fault, spin)) {
            // A copy did not land in time: the fault word is set. Wait (with
            // the full bound) for this stage's copy and the other stage's so
            // none is left writing this CTA's shared memory, then leave.
            mbar_wait(&bars[s], (i >> 1) & 1u, nullptr);
            if (b + stride < batches) mbar_wait(&bars[s ^ 1u], ((i + 1) >> 1) & 1u, nullptr);
            return;
        }
        const Batch bt = locate_batch<R>(a, b);
        // The batch's segments' stream pointers, once a batch: non-gated one
        // segment (the member's rows from bt.local); gated the gate run at
        // slot 0 and the up run at slot R/2.
        const uint8_t* seg[2][F::kStreams];
        {
            const MemberArgs& m0 = gated ? a.member[0] : a.member[bt.member];
#pragma unroll
            for (int q = 0; q < F::kStreams; ++q) {
                const uint64_t off = RowStreams<F>::base(q, m0.blocks) +
                                     static_cast<uint64_t>(m0.first_row + bt.local) * rb[q];
                seg[0][q] = stage + reg[q] + static_cast<uint32_t>(off & 15ull);
            }
            if (gated) {
                const MemberArgs& m1 = a.member[1];
#pragma unroll
                for (int q = 0; q < F::kStreams; ++q) {
                    const uint64_t off = RowStreams<F>::base(q, m1.blocks) +
                                         static_cast<uint64_t>(m1.first_row + bt.local) * rb[q];
                    seg[1][q] = stage + reg[q] + (R > 1 ? R / 2 : 0) * sl[q] + static_cast<uint32_t>(off & 15ull);
                }
            }
        }
        if constexpr (R == 1) {
            // One row a batch: the smallest products, spread over the most warps.
            float acc = 0.0f;
            for (uint32_t g = lo; g < hi; ++g) {
                F A;
                A.load(seg[0], g);
                chain_group1d<F>(A, xl + (g - lo) * 16u, acc, std::make_integer_sequence<int, 32>{});
            }
            red[lane] = acc;
        } else if (kRowsTogether<F, R> && R * W <= 64 && !gated) {   // (R = 8 at 16 warps would spill)
            // Every pair's chain advanced together, k outermost: one read of x
            // (doubled) serves all R/2 pairs, and the pairs' fmas are
            // independent, so a warp has R/2 accumulations in flight at
            // every step. Slots past the live rows read stale stage bytes;
            // their sums are never written.
            float2 acc[R / 2];
#pragma unroll
            for (int p = 0; p < R / 2; ++p) acc[p] = make_float2(0.0f, 0.0f);
            for (uint32_t g = lo; g < hi; ++g) {
                F A[R / 2], B[R / 2];
#pragma unroll
                for (int p = 0; p < R / 2; ++p) {
                    const uint8_t* pa[F::kStreams];
                    const uint8_t* pb[F::kStreams];
#pragma unroll
                    for (int q = 0; q < F::kStreams; ++q) {
                        pa[q] = seg[0][q] + (2u * p) * rb[q];
                        pb[q] = pa[q] + rb[q];
                    }
                    A[p].load(pa, g);
                    B[p].load(pb, g);
                }
                chain_group_rows<F, R / 2>(A, B, xl + (g - lo) * 16u, acc, std::make_integer_sequence<int, 32>{});
            }
#pragma unroll
            for (int p = 0; p < R / 2; ++p) {
                red[(2 * p) * kRedStride + lane] = acc[p].x;
                red[(2 * p + 1) * kRedStride + lane] = acc[p].y;
            }
        } else {
        // Pairs of slots: non-gated rows (2p, 2p+1) of the segment. Gated:
        // with R = 2 the pair is the output's gate row and up row; otherwise
        // pairs p < R/4 are gate rows (2p, 2p+1), then the same up rows. The
        // pairs unrolled, so a warp has R/2 independent chains in flight.
#pragma unroll
        for (int p = 0; p < R / 2; ++p) {
            const bool upper = gated && R > 2 && p >= R / 4;
            const uint32_t ia = upper ? 2u * p - R / 2 : 2u * p;
            const bool la = ia < bt.live;
            const bool lb = (gated && R == 2) ? la : ia + 1u < bt.live;
            const uint8_t* pa[F::kStreams];
            const uint8_t* pb[F::kStreams];
#pragma unroll
            for (int q = 0; q < F::kStreams; ++q) {
                pa[q] = (upper ? seg[1][q] : seg[0][q]) + ia * rb[q];
                pb[q] = (gated && R == 2) ? seg[1][q] : pa[q] + rb[q];
            }
            float2 acc = make_float2(0.0f, 0.0f);   // rows a, b
            for (uint32_t g = lo; g < hi; ++g) {
                F A, B;
                if (la) A.load(pa, g); else A.zero();
                if (lb) B.load(pb, g); else B.zero();
                chain_group2<F>(A, B, xl + (g - lo) * 16u, acc, std::make_integer_sequence<int, 32>{});
            }
            red[(2 * p) * kRedStride + lane] = acc.x;
            red[(2 * p + 1) * kRedStride + lane] = acc.y;
        }
        }
        // The stage is read: let the copy engine refill it with batch i+2
        // (the fence orders these reads before the copy's writes).
        const bool refill = b + 2u * stride < batches;
        if (refill) fence_proxy_async();
        __syncwarp();
        if (refill) issue_batch<F, R>(a, b + 2u * stride, stage, &bars[s], G, lane);
        // Slot `lane`'s total: its 32 range sums added in order (slot_total, :237).
        float total = 0.0f;
        if (lane < static_cast<uint32_t>(R)) {
            const float4* rs = reinterpret_cast<const float4*>(red + lane * kRedStride);
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
                const uint32_t o = a.member[0].out_offset + bt.local + lane;
                a.out[0][static_cast<size_t>(t) * a.out_stride[0] + o] = activate(a.activation, total) * up;
            }
        } else if (lane < bt.live) {
            const MemberArgs& m = a.member[bt.member];
            const uint32_t o = m.out_offset + bt.local + lane;
            if (a.epilogue == kWrite) {
                a.out[0][static_cast<size_t>(t) * a.out_stride[0] + o] = total;
            } else if (a.epilogue == kQKV) {
                a.out[bt.member][static_cast<size_t>(t) * a.out_stride[bt.member] + o] = total;
            } else {   // kGatedByInput (matmul.wgsl:346-350)
                const float u = a.gate_input[static_cast<size_t>(a.token + t) * a.gate_input_stride +
                                             a.gate_input_column + o];
                a.out[0][static_cast<size_t>(t) * a.out_stride[0] + o] = activate(a.activation, total) * u;
            }
        }
        __syncwarp();
    }
}

// ---- several tokens a weight pass ------------------------------------------
// The same warp layout with R = 2 or 4 rows a batch (a pair of rows, or a
// gated output's gate and up rows; or two pairs: four rows, or two outputs'
// gate rows then their up rows) and MT tokens: each weight is decoded once and multiplied
// into MT chains, one per token, each still the reference's chain for that
// (row, token). Tokens go in pairs through the paired FMA (fma.rn.f32x2,
// each half one fma, so each chain keeps its bits): one paired fma advances
// tokens 2p and 2p + 1 of a row, with the row's weight as both halves of one
// operand. x is staged range-major by token pair, the pair's two floats of
// each k side by side; with two pairs each read of x serves both, halving the
// shared-memory traffic a fma. The R·MT range-sum rows meet in shared
// memory, and lane slot·MT + i adds row `slot`'s range sums for token i in
// range order.
template <typename F, int MT, int RP, int k>
__device__ __forceinline__ void chain_step_mt(const F (&A)[RP], const F (&B)[RP], const typename F::Consts2 (&c)[RP],
                                              const float4* x2, uint32_t pair4, float2 (&pa)[RP][MT / 2],
                                              float2 (&pb)[RP][MT / 2]) {
    float2 wa[RP], wb[RP];
#pragma unroll
    for (int r = 0; r < RP; ++r) {
        const float2 w = F::template weight2<k>(A[r], B[r], c[r]);
        wa[r] = make_float2(w.x, w.x);
        wb[r] = make_float2(w.y, w.y);
    }
#pragma unroll
    for (int p = 0; p < MT / 2; ++p) {
        const float4 xq = x2[p * pair4 + k / 2];
        const float2 xk = (k % 2 == 0) ? make_float2(xq.x, xq.y) : make_float2(xq.z, xq.w);
#pragma unroll
        for (int r = 0; r < RP; ++r) {
            pa[r][p] = __ffma2_rn(wa[r], xk, pa[r][p]);
            pb[r][p] = __ffma2_rn(wb[r], xk, pb[r][p]);
        }
    }
}

template <typename F, int MT, int RP, int... ks>
__device__ __forceinline__ void chain_group_mt(const F (&A)[RP], const F (&B)[RP], const float4* x2, uint32_t pair4,
                                               float2 (&pa)[RP][MT / 2], float2 (&pb)[RP][MT / 2],
                                               std::integer_sequence<int, ks...>) {
    typename F::Consts2 c[RP];
#pragma unroll
    for (int r = 0; r < RP; ++r) c[r] = F::consts2(A[r], B[r]);
    (chain_step_mt<F, MT, RP, ks>(A, B, c, x2, pair4, pa, pb), ...);
}

template <typename F, int MT, int W, int R>
__global__ void __launch_bounds__(W * 32) decode_mt_kernel(const MatmulArgs a) {
    static_assert(R == 2 || R == 4, "one or two pairs of rows a batch");
    static_assert(R * MT <= 32, "a batch's totals take one lane each");
    constexpr int RP = R / 2;
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t G = a.columns / 32u;
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t lane_stride = x2_lane_stride(G);
    const uint32_t pair_floats = 32u * lane_stride;   // one token pair's staged x
    const uint32_t stage_bytes = RowStreams<F>::row_stage(G) * R;
    const uint32_t batches = batch_count<R>(a);
    const uint32_t stride = gridDim.x * W;
    const bool gated = a.epilogue == kGated;
    const uint32_t spin = spin_limit_of(a.fault);   // read early: off the first wait's path

    float* xs = reinterpret_cast<float*>(smem);
    const uint32_t x_bytes = MT / 2 * pair_floats * 4u;
    const uint32_t warp_bytes = 16u + R * MT * kRedStride * 4u + 2u * stage_bytes;
    uint8_t* wbase = smem + x_bytes + warp * warp_bytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(wbase);
    float* red = reinterpret_cast<float*>(wbase + 16);
    uint8_t* stages = wbase + 16u + R * MT * kRedStride * 4u;

    if (lane == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        fence_barrier_init();
    }
    __syncwarp();
    const uint32_t first = blockIdx.x * W + warp;
    if (first < batches) issue_batch<F, R>(a, first, stages, &bars[0], G, lane);
    if (first + stride < batches) issue_batch<F, R>(a, first + stride, stages + stage_bytes, &bars[1], G, lane);

    grid_dependency_wait();

    const uint32_t t0 = blockIdx.y * MT;
    const uint32_t nt = min(static_cast<uint32_t>(MT), a.tokens - t0);
    const uint32_t lo = range_lo(lane, G), hi = range_lo(lane + 1u, G);
    // A token pair's 16-byte chunks dealt to all threads in row order (each
    // warp reads one contiguous span of both rows) and interleaved into
    // their range's run; tokens past the step's last are zeros.
    {
        const uint32_t chunks = G * 8u;
        const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
        for (uint32_t idx = threadIdx.x; idx < MT / 2 * chunks; idx += W * 32u) {
            const uint32_t p = idx / chunks, c = idx % chunks;
            const uint32_t grp = c / 8u, lr = lane_of(grp, G);
            const uint32_t i0 = 2u * p;
            const float4 v0 = i0 < nt ? __ldcg(reinterpret_cast<const float4*>(a.x + static_cast<size_t>(t0 + i0) * a.x_stride) + c) : zero;
            const float4 v1 = i0 + 1u < nt ? __ldcg(reinterpret_cast<const float4*>(a.x + static_cast<size_t>(t0 + i0 + 1u) * a.x_stride) + c) : zero;
            float4* dst = reinterpret_cast<float4*>(xs + p * pair_floats + lr * lane_stride + (grp - range_lo(lr, G)) * 64u +
                                                    (c % 8u) * 8u);
            dst[0] = make_float4(v0.x, v1.x, v0.y, v1.y);
            dst[1] = make_float4(v0.z, v1.z, v0.w, v1.w);
        }
    }
    __syncthreads();
    grid_dependents_launch();
    const float4* xl = reinterpret_cast<const float4*>(xs + lane * lane_stride);
    const uint32_t pair4 = pair_floats / 4u;

    uint32_t rb[F::kStreams], sl[F::kStreams], reg[F::kStreams];
#pragma unroll
    for (int q = 0; q < F::kStreams; ++q) {
        rb[q] = RowStreams<F>::row_bytes(q, G);
        sl[q] = RowStreams<F>::slot(q, G);
        reg[q] = q == 0 ? 0u : reg[q - 1] + R * sl[q - 1];
    }

    uint32_t it = 0;
    for (uint32_t b = first; b < batches; b += stride, ++it) {
        const uint32_t s = it & 1u;
        uint8_t* stage = stages + s * stage_bytes;
        if (!mbar_wait(&bars[s], (it >> 1) & 1u, a.fault, spin)) {
            mbar_wait(&bars[s], (it >> 1) & 1u, nullptr);
            if (b + stride < batches) mbar_wait(&bars[s ^ 1u], ((it + 1) >> 1) & 1u, nullptr);
            return;
        }
        const Batch bt = locate_batch<R>(a, b);
        // Stream pointers of the batch's slots: non-gated, rows 0..R-1 of one
        // segment; gated, R = 2: the gate row at slot 0 and the up row at
        // slot 1; R = 4: the gate rows at slots 0 and 1, the up rows at 2 and 3.
        // Pair r is slots (2r, 2r + 1).
        const uint8_t* pa[RP][F::kStreams];
        const uint8_t* pb[RP][F::kStreams];
        {
            const MemberArgs& m0 = gated ? a.member[0] : a.member[bt.member];
            const MemberArgs& m1 = a.member[gated ? 1 : bt.member];
#pragma unroll
            for (int q = 0; q < F::kStreams; ++q) {
                const uint64_t off0 = RowStreams<F>::base(q, m0.blocks) +
                                      static_cast<uint64_t>(m0.first_row + bt.local) * rb[q];
                const uint8_t* s0 = stage + reg[q] + static_cast<uint32_t>(off0 & 15ull);
                if (!gated) {
#pragma unroll
                    for (int r = 0; r < RP; ++r) {
                        pa[r][q] = s0 + (2u * r) * rb[q];
                        pb[r][q] = s0 + (2u * r + 1u) * rb[q];
                    }
                } else {
                    const uint64_t off1 = RowStreams<F>::base(q, m1.blocks) +
                                          static_cast<uint64_t>(m1.first_row + bt.local) * rb[q];
                    const uint8_t* s1 = stage + reg[q] + (R / 2) * sl[q] + static_cast<uint32_t>(off1 & 15ull);
                    if (R == 2) {
                        pa[0][q] = s0;
                        pb[0][q] = s1;
                    } else {
                        pa[0][q] = s0;
                        pb[0][q] = s0 + rb[q];
                        pa[RP - 1][q] = s1;
                        pb[RP - 1][q] = s1 + rb[q];
                    }
                }
            }
        }
        const bool la = bt.live > 0;
        const bool lb = gated ? la : bt.live > 1;
        float2 aa[RP][MT / 2], ab[RP][MT / 2];
#pragma unroll
        for (int r = 0; r < RP; ++r)
#pragma unroll
            for (int p = 0; p < MT / 2; ++p) { aa[r][p] = make_float2(0.0f, 0.0f); ab[r][p] = make_float2(0.0f, 0.0f); }
        for (uint32_t g = lo; g < hi; ++g) {
            F A[RP], B[RP];
            if (R == 2) {
                if (la) A[0].load(pa[0], g); else A[0].zero();
                if (lb) B[0].load(pb[0], g); else B[0].zero();
            } else {
                // Slots past the live rows read stale stage bytes; their sums
                // are never written.
#pragma unroll
                for (int r = 0; r < RP; ++r) {
                    A[r].load(pa[r], g);
                    B[r].load(pb[r], g);
                }
            }
            chain_group_mt<F, MT, RP>(A, B, xl + (g - lo) * 16u, pair4, aa, ab, std::make_integer_sequence<int, 32>{});
        }
#pragma unroll
        for (int r = 0; r < RP; ++r)
#pragma unroll
            for (int p = 0; p < MT / 2; ++p) {
                red[((2 * r) * MT + 2 * p) * kRedStride + lane] = aa[r][p].x;
                red[((2 * r) * MT + 2 * p + 1) * kRedStride + lane] = aa[r][p].y;
                red[((2 * r + 1) * MT + 2 * p) * kRedStride + lane] = ab[r][p].x;
                red[((2 * r + 1) * MT + 2 * p + 1) * kRedStride + lane] = ab[r][p].y;
            }
        fence_proxy_async();
        __syncwarp();
        if (b + 2u * stride < batches) issue_batch<F, R>(a, b + 2u * stride, stage, &bars[s], G, lane);
        // Lane slot·MT + i: row `slot`, token i, its 32 range sums in order.
        float total = 0.0f;
        if (lane < static_cast<uint32_t>(R * MT)) {
            const float4* rs = reinterpret_cast<const float4*>(red + lane * kRedStride);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float4 v = rs[q];
                total = total + v.x;
                total = total + v.y;
                total = total + v.z;
                total = total + v.w;
            }
        }
        const uint32_t slot = lane / MT, ti = lane % MT;
        const uint32_t t = t0 + ti;
        if (gated) {
            const float up = __shfl_down_sync(0xFFFFFFFFu, total, (R / 2) * MT);
            if (slot < static_cast<uint32_t>(R / 2) && slot < bt.live && ti < nt) {
                const uint32_t o = a.member[0].out_offset + bt.local + slot;
                a.out[0][static_cast<size_t>(t) * a.out_stride[0] + o] = activate(a.activation, total) * up;
            }
        } else if (slot < min(bt.live, static_cast<uint32_t>(R)) && lane < static_cast<uint32_t>(R * MT) && ti < nt) {
            const MemberArgs& m = a.member[bt.member];
            const uint32_t o = m.out_offset + bt.local + slot;
            if (a.epilogue == kWrite) {
                a.out[0][static_cast<size_t>(t) * a.out_stride[0] + o] = total;
            } else if (a.epilogue == kQKV) {
                a.out[bt.member][static_cast<size_t>(t) * a.out_stride[bt.member] + o] = total;
            } else {   // kGatedByInput (matmul.wgsl:346-350)
                const float u = a.gate_input[static_cast<size_t>(a.token + t) * a.gate_input_stride +
                                             a.gate_input_column + o];
                a.out[0][static_cast<size_t>(t) * a.out_stride[0] + o] = activate(a.activation, total) * u;
            }
        }
        __syncwarp();
    }
}

template <typename F, int MT, int W = kWarps, int R = 2>
size_t decode_mt_smem(uint32_t G) {
    return static_cast<size_t>(MT / 2) * 32u * x2_lane_stride(G) * 4u +
           W * (16u + static_cast<size_t>(R) * MT * kRedStride * 4u + 2ull * R * RowStreams<F>::row_stage(G));
}

template <typename F, int MT, int W, int R>
cudaError_t launch_decode_mt(const MatmulArgs& a, int sm_count, cudaStream_t stream, bool pdl) {
    const uint32_t G = a.columns / 32u;
    const size_t smem = decode_mt_smem<F, MT, W, R>(G);
    if (smem > static_cast<size_t>(kMaxDecodeSmem)) return cudaErrorInvalidValue;
    uint32_t batches = 0;
    if (a.epilogue == kGated) batches = (a.member[0].rows + R / 2 - 1) / (R / 2);
    else for (uint32_t m = 0; m < a.members; ++m) batches += (a.member[m].rows + R - 1) / R;
    auto kernel = decode_mt_kernel<F, MT, W, R>;
    static bool configured = false;   // per instantiation
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDecodeSmem);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    // CTAs an SM holds at this width (shared memory and registers), per
    // instantiation for the last width asked.
    static size_t occupancy_smem = 0;
    static uint32_t per_sm = 1;
    if (occupancy_smem != smem) {
        int n = 0;
        cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, W * 32, smem);
        if (e != cudaSuccess) return e;
        per_sm = n > 0 ? static_cast<uint32_t>(n) : 1u;
        occupancy_smem = smem;
    }
    const uint32_t groups = (a.tokens + MT - 1) / MT;
    uint32_t ctas = (batches + W - 1) / W;
    // Enough CTAs across the token groups to fill the SMs in one wave, no
    // more: a CTA past the wave would start only when one ends.
    const uint32_t cap = static_cast<uint32_t>(sm_count) * per_sm / groups;
    if (ctas > cap) ctas = cap;
    if (ctas == 0) ctas = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctas, groups);
    cfg.blockDim = dim3(W * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, a);
}

// Tokens a weight pass: 2, 4, 8 or 16 — the fewest that cover a short step,
// 16 for longer ones — stepping down while x of that many tokens and the
// stages do not fit shared memory (wide rows).
// Eight warps a CTA where they fit (x is staged once a CTA, so more warps
// share it), else four. Up to 8 tokens a pass, batches of two pairs of rows
// (each read of x serves both pairs) for the formats whose decoded state
// fits registers for both (kRowsTogether).
template <typename F, int MT, int R>
cudaError_t launch_mt_warps(const MatmulArgs& a, int sm_count, cudaStream_t stream, bool pdl) {
    const uint32_t G = a.columns / 32u;
    if (decode_mt_smem<F, MT, 8, R>(G) <= static_cast<size_t>(kMaxDecodeSmem))
        return launch_decode_mt<F, MT, 8, R>(a, sm_count, stream, pdl);
    return launch_decode_mt<F, MT, 4, R>(a, sm_count, stream, pdl);
}

// Two pairs a batch halve the batches (and the CTAs of a product that fills
// less than a wave) and raise the registers a thread, so they are taken
// where the product is large enough to keep every SM busy either way
// (measured on Gemma-3-1B and Qwen3-0.6B shapes at 2-16 tokens, B200): the
// vocabulary heads at any token count, products of 2,048 slots or more at 8
// tokens, non-gated ones of 4,096 rows or more at 2-4 tokens.
template <typename F, int MT>
cudaError_t launch_mt_rows(const MatmulArgs& a, int sm_count, cudaStream_t stream, bool pdl) {
    constexpr bool two_pairs = MT <= 8 && kRowsTogether<F, 4>;
    const bool gated = a.epilogue == kGated;
    const uint64_t slots = gated ? 2ull * a.member[0].rows : a.total_rows;
    const bool large = slots >= 65536u || (MT == 8 && slots >= 2048u) || (MT <= 4 && !gated && slots >= 4096u);
    if (two_pairs && large &&
        decode_mt_smem<F, MT, 4, two_pairs ? 4 : 2>(a.columns / 32u) <= static_cast<size_t>(kMaxDecodeSmem))
        return launch_mt_warps<F, MT, two_pairs ? 4 : 2>(a, sm_count, stream, pdl);
    return launch_mt_warps<F, MT, 2>(a, sm_count, stream, pdl);
}

template <typename F>
cudaError_t dispatch_mt(const MatmulArgs& a, int sm_count, cudaStream_t stream, bool pdl) {
    const uint32_t G = a.columns / 32u;
    const size_t budget = static_cast<size_t>(kMaxDecodeSmem);
    const uint32_t want = a.tokens > 8 ? 16u : (a.tokens > 4 ? 8u : (a.tokens > 2 ? 4u : 2u));
    if (want >= 16 && decode_mt_smem<F, 16>(G) <= budget) return launch_mt_rows<F, 16>(a, sm_count, stream, pdl);
    if (want >= 8 && decode_mt_smem<F, 8>(G) <= budget) return launch_mt_rows<F, 8>(a, sm_count, stream, pdl);
    if (want >= 4 && decode_mt_smem<F, 4>(G) <= budget) return launch_mt_rows<F, 4>(a, sm_count, stream, pdl);
    if (decode_mt_smem<F, 2>(G) <= budget) return launch_mt_rows<F, 2>(a, sm_count, stream, pdl);
    return cudaErrorInvalidValue;
}

template <typename F, int R, int W = kWarps>
size_t decode_smem(uint32_t G) {
    return 32ull * x2_lane_stride(G) * 4u + W * (16u + R * kRedStride * 4u + 2ull * R * RowStreams<F>::row_stage(G));
}

template <typename F, int R, int W = kWarps>
cudaError_t launch_decode(const MatmulArgs& a, int sm_count, cudaStream_t stream, bool pdl) {
    const uint32_t G = a.columns / 32u;
    const size_t smem = decode_smem<F, R, W>(G);
    if (smem > static_cast<size_t>(kMaxDecodeSmem)) return cudaErrorInvalidValue;
    uint32_t batches = 0;
    if (a.epilogue == kGated) batches = (a.member[0].rows + (R > 1 ? R / 2 : 1) - 1) / (R > 1 ? R / 2 : 1);
    else for (uint32_t m = 0; m < a.members; ++m) batches += (a.member[m].rows + R - 1) / R;
    auto kernel = decode_kernel<F, R, W>;
    static bool configured = false;   // per instantiation
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDecodeSmem);
        if (e != cudaSuccess) return e;
        // The whole unified L1/shared carveout to shared memory, so that
        // launches of different sizes never flip the SM's configuration.
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    uint32_t ctas = (batches + W - 1) / W;
    // Resident CTAs an SM holds at this shared-memory size, times the SMs:
    // beyond that the warps stride over batches with their copies in flight.
    uint32_t per_sm = static_cast<uint32_t>((227u * 1024u) / (smem + 1024u));
    if (per_sm < 1) per_sm = 1;
    if (per_sm > 16) per_sm = 16;
    const uint32_t cap = static_cast<uint32_t>(sm_count) * per_sm;
    if (ctas > cap) ctas = cap;
    if (ctas == 0) ctas = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctas, a.tokens ? a.tokens : 1u);
    cfg.blockDim = dim3(W * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, a);
}

// Latency shape, for products small enough that one batch a warp and at
// most one CTA an SM hold all of their rows: every copy is issued before the
// wait on the grid before, every CTA fits beside that grid's (none starts
// late, when the one before has exited), and x is read once an SM. The
// fewest rows a batch that fit, from two (rows in pairs take the paired
// FMAs), then the fewest warps a CTA (the most SMs).
constexpr size_t kLatencySmem = 100u * 1024u;

template <typename F, int R>
bool latency_shape(const MatmulArgs& a, int sm_count, cudaStream_t stream, bool pdl, cudaError_t& err) {
    const uint32_t G = a.columns / 32u;
    uint64_t batches = 0;
    constexpr uint32_t H = R > 1 ? R / 2 : 1;   // a gated batch's outputs (gated products take R >= 2)
    if (a.epilogue == kGated) batches = (a.member[0].rows + H - 1) / H;
    else for (uint32_t m = 0; m < a.members; ++m) batches += (a.member[m].rows + R - 1) / R;
    const uint64_t sms = static_cast<uint64_t>(sm_count);
    if ((batches + 3) / 4 <= sms && decode_smem<F, R, 4>(G) <= kLatencySmem) {
        err = launch_decode<F, R, 4>(a, sm_count, stream, pdl);
        return true;
    }
    if ((batches + 7) / 8 <= sms && decode_smem<F, R, 8>(G) <= kLatencySmem) {
        err = launch_decode<F, R, 8>(a, sm_count, stream, pdl);
        return true;
    }
    if ((batches + 15) / 16 <= sms && decode_smem<F, R, 16>(G) <= kLatencySmem) {
        err = launch_decode<F, R, 16>(a, sm_count, stream, pdl);
        return true;
    }
    return false;
}

// Rows a batch takes: the latency shape where it fits; otherwise enough
// batches that every SM has several warps, more rows a warp when the
// product is large (fewer, longer copies), fewer rows when a wide row's
// stages would not fit shared memory.
template <typename F>
cudaError_t dispatch(const MatmulArgs& a, int sm_count, cudaStream_t stream, bool pdl) {
    const uint32_t G = a.columns / 32u;
    const bool gated = a.epilogue == kGated;
    cudaError_t err = cudaSuccess;
    if (latency_shape<F, 2>(a, sm_count, stream, pdl, err)) return err;
    if (latency_shape<F, 4>(a, sm_count, stream, pdl, err)) return err;
    if (latency_shape<F, 8>(a, sm_count, stream, pdl, err)) return err;
    const uint64_t slots = gated ? 2ull * a.member[0].rows : a.total_rows;
    const uint64_t warps_wanted = static_cast<uint64_t>(sm_count) * 16u;
    const size_t budget = 110u * 1024u;   // two CTAs an SM at least
    if (slots >= warps_wanted * 8u && decode_smem<F, 8>(G) <= budget) return launch_decode<F, 8>(a, sm_count, stream, pdl);
    if (slots >= warps_wanted * 4u && decode_smem<F, 4>(G) <= budget) return launch_decode<F, 4>(a, sm_count, stream, pdl);
    if (slots >= warps_wanted * 2u || gated) return launch_decode<F, 2>(a, sm_count, stream, pdl);
    return launch_decode<F, 1>(a, sm_count, stream, pdl);
}

}  // namespace

size_t matmul_decode_smem_bytes(uint32_t format, uint32_t columns) {
    const uint32_t G = columns / 32u;
    switch (format) {
        case kQ4_0: return decode_smem<Q4_0, 1>(G);
        case kQ8_0: return decode_smem<Q8_0, 1>(G);
        case kQ6_K: return decode_smem<Q6_K, 1>(G);
        case kQ4_1: return decode_smem<Q4_1, 1>(G);
        case kBF16: return decode_smem<BF16, 1>(G);
        default: return 0;
    }
}

cudaError_t matmul_decode(const MatmulArgs& a, int sm_count, cudaStream_t stream, bool pdl) {
    if (a.tokens > 1) {
        switch (a.format) {
            case kQ4_0: return dispatch_mt<Q4_0>(a, sm_count, stream, pdl);
            case kQ8_0: return dispatch_mt<Q8_0>(a, sm_count, stream, pdl);
            case kQ6_K: return dispatch_mt<Q6_K>(a, sm_count, stream, pdl);
            case kQ4_1: return dispatch_mt<Q4_1>(a, sm_count, stream, pdl);
            case kBF16: return dispatch_mt<BF16>(a, sm_count, stream, pdl);
            default: return cudaErrorInvalidValue;
        }
    }
    switch (a.format) {
        case kQ4_0: return dispatch<Q4_0>(a, sm_count, stream, pdl);
        case kQ8_0: return dispatch<Q8_0>(a, sm_count, stream, pdl);
        case kQ6_K: return dispatch<Q6_K>(a, sm_count, stream, pdl);
        case kQ4_1: return dispatch<Q4_1>(a, sm_count, stream, pdl);
        case kBF16: return dispatch<BF16>(a, sm_count, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace cb
