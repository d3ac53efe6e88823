// Building blocks of the decode GEMV shared by the decode kernels and the
// fused decode step: the reference's 32 ranges (plainsight-systems/charlotte,
// src/core/kernels/matmul/matmul.wgsl decode_ranges :212, slot_total :237;
// matmul.h:34-50), batches of rows a warp owns, their bulk copies into a
// warp's shared stage, and the fma chains of a group. The arithmetic of an
// output is fixed here, so every kernel built from these gives it the same
// bits.
#pragma once

#include <cstdint>
#include <utility>

#include "formats.cuh"
#include "matmul.h"
#include "tma.cuh"

namespace cb {

constexpr int kRedStride = 36;   // floats per row of range sums (16-byte rows, conflict-free float4 reads)

__host__ __device__ __forceinline__ uint32_t range_lo(uint32_t r, uint32_t G) { return r * G / 32u; }

// The lane whose range holds group g: the largest r with floor(r·G/32) <= g.
__device__ __forceinline__ uint32_t lane_of(uint32_t g, uint32_t G) { return (32u * (g + 1u) + G - 1u) / G - 1u; }

// Floats of x a range holds in shared memory: its most groups, and a 16-byte skew.
__host__ __device__ __forceinline__ uint32_t x_lane_stride(uint32_t G) { return (G + 31u) / 32u * 32u + 4u; }

// The same with every float of x held twice ((x_k, x_k), the paired FMA's
// operand for two rows): a group takes 64 floats; the 16-byte skew keeps a
// quarter-warp's 16-byte reads on distinct banks.
__host__ __device__ __forceinline__ uint32_t x2_lane_stride(uint32_t G) { return (G + 31u) / 32u * 64u + 4u; }

// A batch: up to R consecutive rows of one member (non-gated), or R/2
// outputs' gate rows then the same up rows (gated). Batches never straddle
// members, so a batch's rows of each stream are one contiguous run.
struct Batch {
    uint32_t member;   // non-gated: the member; gated: 0
    uint32_t local;    // first row's index within the member's rows (gated: first output)
    uint32_t live;     // rows live (gated: outputs live)
};

template <int R>
__device__ __forceinline__ uint32_t batch_count(const MatmulArgs& a) {
    if (a.epilogue == kGated) return (a.member[0].rows + (R > 1 ? R / 2 : 1) - 1) / (R > 1 ? R / 2 : 1);
    uint32_t n = 0;
    for (uint32_t m = 0; m < a.members; ++m) n += (a.member[m].rows + R - 1) / R;
    return n;
}

template <int R>
__device__ __forceinline__ Batch locate_batch(const MatmulArgs& a, uint32_t b) {
    Batch r{0, 0, 0};
    if (a.epilogue == kGated) {
        constexpr uint32_t H = R > 1 ? R / 2 : 1;
        r.local = b * H;
        r.live = min(H, a.member[0].rows - r.local);
        return r;
    }
    for (uint32_t m = 0; m < a.members; ++m) {
        const uint32_t nb = (a.member[m].rows + R - 1) / R;
        if (b < nb) {
            r.member = m;
            r.local = b * R;
            r.live = min(static_cast<uint32_t>(R), a.member[m].rows - r.local);
            return r;
        }
        b -= nb;
    }
    return r;
}

// The stage is stream-major: stream s's region holds R slots of
// RowStreams<F>::slot(s) bytes. A run of consecutive rows (a segment) is one
// bulk copy per stream, rounded out to 16-byte bounds, at the region's slot
// `j0`; its row i lies (off mod 16) + i·row_bytes past that.
template <typename F>
struct Stage {
    __device__ __forceinline__ static uint32_t region(int s, uint32_t G, int R) {
        uint32_t at = 0;
        for (int t = 0; t < s; ++t) at += R * RowStreams<F>::slot(t, G);
        return at;
    }
    __device__ __forceinline__ static uint32_t copy_segment(uint8_t* stage, const MemberArgs& m, uint32_t row,
                                                            uint32_t j0, uint32_t len, uint32_t G, int R,
                                                            uint64_t* bar, bool issue) {
        uint32_t bytes = 0;
#pragma unroll
        for (int s = 0; s < F::kStreams; ++s) {
            const uint64_t off = RowStreams<F>::base(s, m.blocks) + static_cast<uint64_t>(row) * RowStreams<F>::row_bytes(s, G);
            const uint64_t start = off & ~15ull;
            const uint64_t end = (off + static_cast<uint64_t>(len) * RowStreams<F>::row_bytes(s, G) + 15ull) & ~15ull;
            if (issue)
                bulk_g2s(stage + region(s, G, R) + j0 * RowStreams<F>::slot(s, G), m.piece + start,
                         static_cast<uint32_t>(end - start), bar);
            bytes += static_cast<uint32_t>(end - start);
        }
        return bytes;
    }
    // Stream pointers of row i of the segment copied at slot j0 from `row`.
    __device__ __forceinline__ static void pointers(const uint8_t* stage, const MemberArgs& m, uint32_t row,
                                                    uint32_t j0, uint32_t i, uint32_t G, int R, const uint8_t** p) {
#pragma unroll
        for (int s = 0; s < F::kStreams; ++s) {
            const uint64_t off = RowStreams<F>::base(s, m.blocks) + static_cast<uint64_t>(row) * RowStreams<F>::row_bytes(s, G);
            p[s] = stage + region(s, G, R) + j0 * RowStreams<F>::slot(s, G) + static_cast<uint32_t>(off & 15ull) +
                   i * RowStreams<F>::row_bytes(s, G);
        }
    }
};

// Issues batch b's copies into `stage`: lane 0 arms the barrier with the
// batch's bytes, then issues one copy per stream per segment (gated: the
// gate run and the up run).
template <typename F, int R>
__device__ __forceinline__ void issue_batch(const MatmulArgs& a, uint32_t b, uint8_t* stage, uint64_t* bar,
                                            uint32_t G, uint32_t lane) {
    if (lane != 0) return;
    const Batch bt = locate_batch<R>(a, b);
    if (a.epilogue == kGated) {
        const MemberArgs& g = a.member[0];
        const MemberArgs& u = a.member[1];
        const uint32_t bytes = Stage<F>::copy_segment(stage, g, g.first_row + bt.local, 0, bt.live, G, R, bar, false) +
                               Stage<F>::copy_segment(stage, u, u.first_row + bt.local, R / 2, bt.live, G, R, bar, false);
        static_assert(R >= 2 || true, "");
        mbar_arrive_expect_tx(bar, bytes);
        Stage<F>::copy_segment(stage, g, g.first_row + bt.local, 0, bt.live, G, R, bar, true);
        Stage<F>::copy_segment(stage, u, u.first_row + bt.local, R / 2, bt.live, G, R, bar, true);
    } else {
        const MemberArgs& m = a.member[bt.member];
        const uint32_t bytes = Stage<F>::copy_segment(stage, m, m.first_row + bt.local, 0, bt.live, G, R, bar, false);
        mbar_arrive_expect_tx(bar, bytes);
        Stage<F>::copy_segment(stage, m, m.first_row + bt.local, 0, bt.live, G, R, bar, true);
    }
}

template <typename F, int k>
__device__ __forceinline__ void chain_step(const F& A, const F& B, const typename F::Consts& ca,
                                           const typename F::Consts& cbb, const float4* x4, float& acc_a,
                                           float& acc_b) {
    const float4 xq = x4[k / 4];
    const float xk = (k % 4 == 0) ? xq.x : ((k % 4 == 1) ? xq.y : ((k % 4 == 2) ? xq.z : xq.w));
    const float wa = F::template weight<k>(A, ca);
    const float wb = F::template weight<k>(B, cbb);
    acc_a = fmaf(wa, xk, acc_a);
    acc_b = fmaf(wb, xk, acc_b);
}

template <typename F, int... ks>
__device__ __forceinline__ void chain_group(const F& A, const F& B, const float4* x4, float& acc_a, float& acc_b,
                                            std::integer_sequence<int, ks...>) {
    const typename F::Consts ca = A.consts(), cbb = B.consts();
    (chain_step<F, ks>(A, B, ca, cbb, x4, acc_a, acc_b), ...);
}

// Two rows' chains as one: each step's decode and multiply-add run as paired
// FMAs (fma.rn.f32x2: two independent fused multiply-adds, each rounded
// once, so each row's bits are those of chain_step). x2 holds x doubled.
template <typename F, int k>
__device__ __forceinline__ void chain_step2(const F& A, const F& B, const typename F::Consts2& c, const float4* x2,
                                            float2& acc) {
    const float4 xq = x2[k / 2];
    const float2 xk = (k % 2 == 0) ? make_float2(xq.x, xq.y) : make_float2(xq.z, xq.w);
    acc = __ffma2_rn(F::template weight2<k>(A, B, c), xk, acc);
}

template <typename F, int... ks>
__device__ __forceinline__ void chain_group2(const F& A, const F& B, const float4* x2, float2& acc,
                                             std::integer_sequence<int, ks...>) {
    const typename F::Consts2 c = F::consts2(A, B);
    (chain_step2<F, ks>(A, B, c, x2, acc), ...);
}

// P pairs of rows at once: step k reads x once (doubled) and advances each
// pair's chain by one paired decode and one paired fma — each row's
// operations and their order those of chain_step2.
template <typename F, int P, int k>
__device__ __forceinline__ void chain_step_rows(const F (&A)[P], const F (&B)[P], const typename F::Consts2 (&c)[P],
                                                const float4* x2, float2 (&acc)[P]) {
    const float4 xq = x2[k / 2];
    const float2 xk = (k % 2 == 0) ? make_float2(xq.x, xq.y) : make_float2(xq.z, xq.w);
#pragma unroll
    for (int p = 0; p < P; ++p) acc[p] = __ffma2_rn(F::template weight2<k>(A[p], B[p], c[p]), xk, acc[p]);
}

template <typename F, int P, int... ks>
__device__ __forceinline__ void chain_group_rows(const F (&A)[P], const F (&B)[P], const float4* x2, float2 (&acc)[P],
                                                 std::integer_sequence<int, ks...>) {
    typename F::Consts2 c[P];
#pragma unroll
    for (int p = 0; p < P; ++p) c[p] = F::consts2(A[p], B[p]);
    (chain_step_rows<F, P, ks>(A, B, c, x2, acc), ...);
}

// One row's chain reading x doubled (x2).
template <typename F, int k>
__device__ __forceinline__ void chain_step1d(const F& A, const typename F::Consts& ca, const float4* x2, float& acc) {
    const float4 xq = x2[k / 2];
    const float xk = (k % 2 == 0) ? xq.x : xq.z;
    acc = fmaf(F::template weight<k>(A, ca), xk, acc);
}

template <typename F, int... ks>
__device__ __forceinline__ void chain_group1d(const F& A, const float4* x2, float& acc,
                                              std::integer_sequence<int, ks...>) {
    const typename F::Consts ca = A.consts();
    (chain_step1d<F, ks>(A, ca, x2, acc), ...);
}

template <typename F, int k>
__device__ __forceinline__ void chain_step1(const F& A, const typename F::Consts& ca, const float4* x4, float& acc) {
    const float4 xq = x4[k / 4];
    const float xk = (k % 4 == 0) ? xq.x : ((k % 4 == 1) ? xq.y : ((k % 4 == 2) ? xq.z : xq.w));
    acc = fmaf(F::template weight<k>(A, ca), xk, acc);
}

template <typename F, int... ks>
__device__ __forceinline__ void chain_group1(const F& A, const float4* x4, float& acc,
                                             std::integer_sequence<int, ks...>) {
    const typename F::Consts ca = A.consts();
    (chain_step1<F, ks>(A, ca, x4, acc), ...);
}


}  // namespace cb
