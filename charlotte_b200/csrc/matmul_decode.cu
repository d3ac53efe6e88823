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
//  - A warp owns batches of R rows (R = 2, 4 or 8, chosen by the product's
//    size so that small products still spread over every SM). Each batch's
//    row streams (codes, scales, ...) are brought into the warp's shared
//    memory by bulk asynchronous copies (cp.async.bulk, the untiled TMA),
//    completing on an mbarrier, through a two-stage ring: the copy of batch
//    i+2 is in flight while batch i is worked.
//  - The first two batches' copies are issued before griddepcontrol.wait:
//    weights are never written on the device, so under programmatic
//    dependent launch a product's weight stream overlaps the launch before it;
//    only x, the previous launch's output, waits.
//  - Rows are worked two at a time sharing each x read: one fma decodes a
//    weight exactly (formats.cuh), one fma accumulates it.
//  - A batch's rows that are consecutive in one weight (all of them, but at
//    a member's edge or the product's end) come in one bulk copy per stream.
//  - x is staged once per CTA in shared memory range-major, a 16-byte skew
//    per range, so the lanes' 128-bit reads fall in distinct banks.
//  - Every mbarrier wait is bounded (tma.cuh): a copy that never lands sets
//    the launch's fault word, which the host reports as a failed step.
#include <cuda_runtime.h>

#include <cstdint>
#include <utility>

#include "formats.cuh"
#include "matmul.h"
#include "numerics.cuh"
#include "tma.cuh"

namespace cb {

namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kRedStride = 36;   // floats per row of range sums (16-byte rows, conflict-free float4 reads)
constexpr int kMaxDecodeSmem = 220 * 1024;

__host__ __device__ __forceinline__ uint32_t range_lo(uint32_t r, uint32_t G) { return r * G / 32u; }

// The lane whose range holds group g: the largest r with floor(r·G/32) <= g.
__device__ __forceinline__ uint32_t lane_of(uint32_t g, uint32_t G) { return (32u * (g + 1u) + G - 1u) / G - 1u; }

// Floats of x a range holds in shared memory: its most groups, and a 16-byte skew.
__host__ __device__ __forceinline__ uint32_t x_lane_stride(uint32_t G) { return (G + 31u) / 32u * 32u + 4u; }

struct Slot {
    const uint8_t* piece;
    uint32_t blocks;
    uint32_t row;     // row within the piece
    uint32_t member;
    uint32_t out;     // output column
    bool live;
};

// Slot s (0..R-1) of batch b. Write/QKV/GatedByInput: the product's rows in
// order, members concatenated. Gated: R/2 outputs a batch, gate rows in slots
// 0..R/2-1 and the same up rows in R/2..R-1.
template <int R>
__device__ __forceinline__ Slot locate_slot(const MatmulArgs& a, uint32_t batch, uint32_t s) {
    Slot r{};
    if (a.epilogue == kGated) {
        constexpr uint32_t H = R / 2;
        const uint32_t m = s / H;
        const uint32_t row = batch * H + (s % H);
        r.member = m;
        r.live = row < a.member[0].rows;
        r.piece = a.member[m].piece;
        r.blocks = a.member[m].blocks;
        r.row = a.member[m].first_row + row;
        r.out = a.member[0].out_offset + row;
        return r;
    }
    uint32_t v = batch * R + s;
    for (uint32_t m = 0; m < a.members; ++m) {
        if (v < a.member[m].rows) {
            r.member = m;
            r.live = true;
            r.piece = a.member[m].piece;
            r.blocks = a.member[m].blocks;
            r.row = a.member[m].first_row + v;
            r.out = a.member[m].out_offset + v;
            return r;
        }
        v -= a.member[m].rows;
    }
    r.live = false;
    r.piece = a.member[0].piece;
    r.blocks = a.member[0].blocks;
    return r;
}

// Whether slot j continues the segment of slot j-1: both live, one member,
// consecutive rows (always so within a member).
__device__ __forceinline__ bool continues(const Slot& prev, const Slot& cur) {
    return prev.live && cur.live && prev.member == cur.member && prev.row + 1u == cur.row;
}

// A batch's stage is stream-major: stream s's region holds R slots of
// RowStreams<F>::slot(s) bytes. A segment of consecutive rows starting at
// slot j0 is one bulk copy per stream, rounded out to 16-byte bounds, placed
// at slot j0 of each region; slot j of the segment then lies
// (off(j0) mod 16) + (j - j0)·row_bytes past that.
template <typename F>
struct Stage {
    __device__ __forceinline__ static uint64_t offset(const Slot& sl, int s, uint32_t G) {
        return RowStreams<F>::base(s, sl.blocks) + static_cast<uint64_t>(sl.row) * RowStreams<F>::row_bytes(s, G);
    }
    __device__ __forceinline__ static uint32_t region(int s, uint32_t G, int R) {
        uint32_t at = 0;
        for (int t = 0; t < s; ++t) at += R * RowStreams<F>::slot(t, G);
        return at;
    }
    // Copies a segment of `len` rows starting at slot j0 (`first` its first row).
    __device__ __forceinline__ static uint32_t copy_segment(uint8_t* stage, const Slot& first, uint32_t j0,
                                                            uint32_t len, uint32_t G, int R, uint64_t* bar,
                                                            bool issue) {
        uint32_t bytes = 0;
#pragma unroll
        for (int s = 0; s < F::kStreams; ++s) {
            const uint64_t off = offset(first, s, G);
            const uint64_t start = off & ~15ull;
            const uint64_t end = (off + static_cast<uint64_t>(len) * RowStreams<F>::row_bytes(s, G) + 15ull) & ~15ull;
            if (issue)
                bulk_g2s(stage + region(s, G, R) + j0 * RowStreams<F>::slot(s, G), first.piece + start,
                         static_cast<uint32_t>(end - start), bar);
            bytes += static_cast<uint32_t>(end - start);
        }
        return bytes;
    }
    // Slot j's stream pointers, given its segment's first slot j0 and row.
    __device__ __forceinline__ static void pointers(const uint8_t* stage, const Slot& first, uint32_t j0, uint32_t j,
                                                    uint32_t G, int R, const uint8_t** p) {
#pragma unroll
        for (int s = 0; s < F::kStreams; ++s)
            p[s] = stage + region(s, G, R) + j0 * RowStreams<F>::slot(s, G) +
                   static_cast<uint32_t>(offset(first, s, G) & 15ull) + (j - j0) * RowStreams<F>::row_bytes(s, G);
    }
};

// Issues batch `batch`'s copies into `stage` (warp-cooperative): lane j < R
// holds slot j; each segment's first lane copies the segment; lane 0 arms
// the barrier with the batch's bytes first.
template <typename F, int R>
__device__ __forceinline__ void issue_batch(const MatmulArgs& a, uint32_t batch, uint8_t* stage, uint64_t* bar,
                                            uint32_t G, uint32_t lane) {
    Slot mine{};
    if (lane < static_cast<uint32_t>(R)) mine = locate_slot<R>(a, batch, lane);
    // The previous slot's member and row, to find segment starts.
    const uint32_t prev_member = __shfl_up_sync(0xFFFFFFFFu, mine.member, 1);
    const uint32_t prev_row = __shfl_up_sync(0xFFFFFFFFu, mine.row, 1);
    const bool prev_live = __shfl_up_sync(0xFFFFFFFFu, mine.live ? 1u : 0u, 1) != 0u && lane > 0;
    const bool cont = lane < static_cast<uint32_t>(R) && mine.live && prev_live && prev_member == mine.member &&
                      prev_row + 1u == mine.row;
    const bool start = lane < static_cast<uint32_t>(R) && mine.live && !cont;
    const uint32_t cont_mask = __ballot_sync(0xFFFFFFFFu, cont);
    // Rows of my segment: me and the run of continuing lanes after me.
    const uint32_t after = ~(cont_mask >> (lane + 1u));
    const uint32_t len = lane < 31u ? 1u + (__ffs(after) - 1u) : 1u;
    uint32_t bytes = start ? Stage<F>::copy_segment(stage, mine, lane, len, G, R, bar, false) : 0u;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) bytes += __shfl_xor_sync(0xFFFFFFFFu, bytes, o);
    if (lane == 0) mbar_arrive_expect_tx(bar, bytes);
    __syncwarp();
    if (start) Stage<F>::copy_segment(stage, mine, lane, len, G, R, bar, true);
}

template <typename F, int k>
__device__ __forceinline__ void chain_step(const F& A, const F& B, const typename F::Consts& ca,
                                           const typename F::Consts& cbb, const float4* x4, float& acc_a,
                                           float& acc_b) {
    const float4 xq = x4[k / 4];
    const float xk = (k % 4 == 0) ? xq.x : ((k % 4 == 1) ? xq.y : ((k % 4 == 2) ? xq.z : xq.w));
    const float wa = fmaf(__uint_as_float(A.template magic<k>()), F::template S<k>(ca), F::template C<k>(ca));
    const float wb = fmaf(__uint_as_float(B.template magic<k>()), F::template S<k>(cbb), F::template C<k>(cbb));
    acc_a = fmaf(wa, xk, acc_a);
    acc_b = fmaf(wb, xk, acc_b);
}

template <typename F, int... ks>
__device__ __forceinline__ void chain_group(const F& A, const F& B, const float4* x4, float& acc_a, float& acc_b,
                                            std::integer_sequence<int, ks...>) {
    const typename F::Consts ca = A.consts(), cbb = B.consts();
    (chain_step<F, ks>(A, B, ca, cbb, x4, acc_a, acc_b), ...);
}

template <typename F, int R>
__global__ void __launch_bounds__(kThreads) decode_kernel(const MatmulArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t G = a.columns / 32u;
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t lane_stride = x_lane_stride(G);
    const uint32_t stage_bytes = RowStreams<F>::row_stage(G) * R;
    const uint32_t batches = a.epilogue == kGated ? (a.member[0].rows + R / 2 - 1) / (R / 2)
                                                  : (a.total_rows + R - 1) / R;
    const uint32_t stride = gridDim.x * kWarps;

    // Shared memory: x (range-major floats), then per warp: 2 barriers,
    // range sums, 2 stages.
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
    const uint32_t first = blockIdx.x * kWarps + warp;
    if (first < batches) issue_batch<F, R>(a, first, stages, &bars[0], G, lane);
    if (first + stride < batches) issue_batch<F, R>(a, first + stride, stages + stage_bytes, &bars[1], G, lane);

    grid_dependency_wait();

    // x, range-major: lane r's groups at r·lane_stride, a 16-byte skew a
    // range; warp w copies the lane's groups w, w+4, ... (no division).
    const uint32_t t = blockIdx.y;
    const uint32_t lo = range_lo(lane, G), hi = range_lo(lane + 1u, G);
    {
        const float4* xg = reinterpret_cast<const float4*>(a.x + static_cast<size_t>(t) * a.x_stride);
        float4* dst = reinterpret_cast<float4*>(xs + lane * lane_stride);
        for (uint32_t g = lo + warp; g < hi; g += kWarps)
#pragma unroll
            for (int v = 0; v < 8; ++v) dst[(g - lo) * 8u + v] = xg[g * 8u + v];
    }
    __syncthreads();
    grid_dependents_launch();
    const float4* xl = reinterpret_cast<const float4*>(xs + lane * lane_stride);

    uint32_t i = 0;
    for (uint32_t batch = first; batch < batches; batch += stride, ++i) {
        const uint32_t s = i & 1u;
        uint8_t* stage = stages + s * stage_bytes;
        if (!mbar_wait(&bars[s], (i >> 1) & 1u, a.fault)) {
            // A copy did not land in time: the fault word is set. Wait (bounded)
            // for the other stage's copy so none is left writing this CTA's
            // shared memory, then leave.
            if (batch + stride < batches) mbar_wait(&bars[s ^ 1u], ((i + 1) >> 1) & 1u, nullptr);
            return;
        }
        // Each slot, its segment's first slot (static indices only).
        Slot sl[R], head[R];
        uint32_t j0[R];
#pragma unroll
        for (int j = 0; j < R; ++j) {
            sl[j] = locate_slot<R>(a, batch, j);
            const bool c = j > 0 && continues(sl[j > 0 ? j - 1 : 0], sl[j]);
            head[j] = c ? head[j > 0 ? j - 1 : 0] : sl[j];
            j0[j] = c ? j0[j > 0 ? j - 1 : 0] : static_cast<uint32_t>(j);
        }
        float acc[R];
#pragma unroll
        for (int p = 0; p < R / 2; ++p) {
            const uint8_t* pa[F::kStreams];
            const uint8_t* pb[F::kStreams];
            Stage<F>::pointers(stage, head[2 * p], j0[2 * p], 2 * p, G, R, pa);
            Stage<F>::pointers(stage, head[2 * p + 1], j0[2 * p + 1], 2 * p + 1, G, R, pb);
            const bool la = sl[2 * p].live, lb = sl[2 * p + 1].live;
            float aa = 0.0f, ab = 0.0f;
            for (uint32_t g = lo; g < hi; ++g) {
                F A, B;
                if (la) A.load(pa, g); else A.zero();
                if (lb) B.load(pb, g); else B.zero();
                chain_group<F>(A, B, xl + (g - lo) * 8u, aa, ab, std::make_integer_sequence<int, 32>{});
            }
            acc[2 * p] = aa;
            acc[2 * p + 1] = ab;
        }
        // The stage is read: let the copy engine refill it with batch i+2.
        fence_proxy_async();
        __syncwarp();
        if (batch + 2u * stride < batches) issue_batch<F, R>(a, batch + 2u * stride, stage, &bars[s], G, lane);
#pragma unroll
        for (int j = 0; j < R; ++j) red[j * kRedStride + lane] = acc[j];
        __syncwarp();
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
        const Slot me = locate_slot<R>(a, batch, lane < static_cast<uint32_t>(R) ? lane : 0u);
        if (a.epilogue == kGated) {
            const float up = __shfl_down_sync(0xFFFFFFFFu, total, R / 2);
            if (lane < static_cast<uint32_t>(R / 2) && me.live)
                a.out[0][static_cast<size_t>(t) * a.out_stride[0] + me.out] = activate(a.activation, total) * up;
        } else if (lane < static_cast<uint32_t>(R) && me.live) {
            if (a.epilogue == kWrite) {
                a.out[0][static_cast<size_t>(t) * a.out_stride[0] + me.out] = total;
            } else if (a.epilogue == kQKV) {
                a.out[me.member][static_cast<size_t>(t) * a.out_stride[me.member] + me.out] = total;
            } else {   // kGatedByInput (matmul.wgsl:346-350)
                const float u = a.gate_input[static_cast<size_t>(a.token + t) * a.gate_input_stride +
                                             a.gate_input_column + me.out];
                a.out[0][static_cast<size_t>(t) * a.out_stride[0] + me.out] = activate(a.activation, total) * u;
            }
        }
        __syncwarp();
    }
}

template <typename F, int R>
size_t decode_smem(uint32_t G) {
    return 32ull * x_lane_stride(G) * 4u + kWarps * (16u + R * kRedStride * 4u + 2ull * R * RowStreams<F>::row_stage(G));
}

template <typename F, int R>
cudaError_t launch_decode(const MatmulArgs& a, int sm_count, cudaStream_t stream, bool pdl) {
    const uint32_t G = a.columns / 32u;
    const size_t smem = decode_smem<F, R>(G);
    if (smem > static_cast<size_t>(kMaxDecodeSmem)) return cudaErrorInvalidValue;
    const uint32_t batches = a.epilogue == kGated ? (a.member[0].rows + R / 2 - 1) / (R / 2)
                                                  : (a.total_rows + R - 1) / R;
    auto kernel = decode_kernel<F, R>;
    static bool configured = false;   // per instantiation
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDecodeSmem);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    uint32_t ctas = (batches + kWarps - 1) / kWarps;
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
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, a);
}

// Rows a batch takes: enough batches that every SM has several warps, more
// rows a warp when the product is large (fewer, longer copies); fewer rows
// when a wide row's stages would not fit shared memory.
template <typename F>
cudaError_t dispatch(const MatmulArgs& a, int sm_count, cudaStream_t stream, bool pdl) {
    const uint32_t G = a.columns / 32u;
    const uint64_t slots = a.epilogue == kGated ? 2ull * a.member[0].rows : a.total_rows;
    const uint64_t warps_wanted = static_cast<uint64_t>(sm_count) * 16u;
    const size_t budget = 110u * 1024u;   // two CTAs an SM at least
    if (slots >= warps_wanted * 8u && decode_smem<F, 8>(G) <= budget) return launch_decode<F, 8>(a, sm_count, stream, pdl);
    if (slots >= warps_wanted * 4u && decode_smem<F, 4>(G) <= budget) return launch_decode<F, 4>(a, sm_count, stream, pdl);
    return launch_decode<F, 2>(a, sm_count, stream, pdl);
}

}  // namespace

size_t matmul_decode_smem_bytes(uint32_t format, uint32_t columns) {
    const uint32_t G = columns / 32u;
    switch (format) {
        case kQ4_0: return decode_smem<Q4_0, 2>(G);
        case kQ8_0: return decode_smem<Q8_0, 2>(G);
        case kQ6_K: return decode_smem<Q6_K, 2>(G);
        default: return 0;
    }
}

cudaError_t matmul_decode(const MatmulArgs& a, int sm_count, cudaStream_t stream, bool pdl) {
    switch (a.format) {
        case kQ4_0: return dispatch<Q4_0>(a, sm_count, stream, pdl);
        case kQ8_0: return dispatch<Q8_0>(a, sm_count, stream, pdl);
        case kQ6_K: return dispatch<Q6_K>(a, sm_count, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace cb
