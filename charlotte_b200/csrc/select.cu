// Top-k selection and the draw (plainsight-systems/charlotte,
// src/core/kernels/topk/topk.wgsl first/merge :131-165, key_of :28,
// before :55; launcher topk.cpp:21; src/core/sampler/draw.wgsl:71-163).
//
// The reference keeps the top 64 of the vocabulary under one total order —
// larger logit first, of equal logits the lower token; −0 = +0; every NaN
// above +∞ — as (logit bits, token) pairs, a NaN's bits canonical
// (0x7FC00000), padding (0xFFFFFFFF, 0xFFFFFFFF) when fewer than 64 exist.
// That order is one comparison here: the 64-bit key
//     key_of(bits) << 32 | (0xFFFFFFFF − token)
// descending, padding 0. Any exact selection of the 64 largest keys gives
// the reference's candidates, in its order.
//
// B200 mapping: one launch. Each CTA takes a tile of 1,024 keys and writes
// its top 64, sorted (bitonic networks in registers: warps sort 32 keys,
// lists of 64 halve by top-64 merges). The last CTA of each group of 16
// tiles to finish (an atomic ticket, no waiting) merges the group's sorted
// lists pairwise by rank; the last group to finish merges the groups' lists
// the same way and runs the draw on the 64 candidates, writing the 16-byte
// sampled record. Tickets (one a group and one overall) are reset for the
// next step.
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"
#include "numerics.cuh"
#include "tma.cuh"

namespace cb {

namespace {

constexpr uint32_t kTile = 1024;
constexpr uint32_t kKeep = 64;
constexpr uint32_t kSelThreads = 1024;
constexpr uint32_t kMaxTiles = 256;   // vocabularies up to 262,144 (the partials a caller provides)
constexpr uint32_t kGroup = 16;       // tiles a first-level merge takes (256 tiles: 16 groups)

__device__ __forceinline__ uint64_t entry_key(uint32_t bits, uint32_t id) {
    return (static_cast<uint64_t>(key_of(bits)) << 32) | static_cast<uint64_t>(0xFFFFFFFFu - id);
}

__device__ __forceinline__ void entry_pair(uint64_t k, uint32_t* out) {
    out[0] = bits_of(static_cast<uint32_t>(k >> 32));
    out[1] = 0xFFFFFFFFu - static_cast<uint32_t>(k);
}

// One compare-exchange of a bitonic network between lanes `lane` and
// `lane ^ j` of a warp (one register each): the lower lane keeps the larger
// key when the run is descending, the smaller when ascending.
__device__ __forceinline__ uint64_t exchange(uint64_t v, uint32_t j, bool descending, uint32_t lane) {
    const uint64_t w = __shfl_xor_sync(0xFFFFFFFFu, v, j);
    return (((lane & j) == 0) == descending) ? (v > w ? v : w) : (v < w ? v : w);
}

// Sorts a bitonic 64-key list held as (r0: positions 0..31, r1: 32..63,
// position = lane + 32·register) descending.
__device__ __forceinline__ void bitonic_merge64(uint64_t& r0, uint64_t& r1, uint32_t lane) {
    const uint64_t hi = r0 > r1 ? r0 : r1, lo = r0 > r1 ? r1 : r0;
    r0 = hi;
    r1 = lo;
#pragma unroll
    for (uint32_t j = 16; j > 0; j >>= 1) {
        r0 = exchange(r0, j, true, lane);
        r1 = exchange(r1, j, true, lane);
    }
}

// The 64 largest of the tile's 1,024 keys (thread t holding `v`, position
// t), sorted descending, into buf[0..63]. Each warp sorts its 32 keys in
// registers (a bitonic sort over the lanes); warp w < 16 joins its list
// with warp w + 16's into a sorted 64; then the lists halve four times,
// warp w keeping the top 64 of its list and list w + n/2's: the larger of
// A[i] and B[63 − i] at each position is a bitonic sequence holding exactly
// the union's top 64, which one bitonic merge sorts. Lists pass through
// `buf` (1,024 keys), one barrier a level.
__device__ void top_of_tile(uint64_t v, uint64_t* buf) {
    const uint32_t t = threadIdx.x, lane = t & 31u, warp = t >> 5;
#pragma unroll
    for (uint32_t k = 2; k <= 32u; k <<= 1)
#pragma unroll
        for (uint32_t j = k >> 1; j > 0; j >>= 1) v = exchange(v, j, (lane & k) == 0, lane);
    if (warp >= 16u) buf[(warp - 16u) * 64u + 32u + lane] = v;
    __syncthreads();
    uint64_t r0 = v, r1 = 0;
    if (warp < 16u) {
        r1 = buf[warp * 64u + 32u + (31u - lane)];   // the other list reversed: ascending
        bitonic_merge64(r0, r1, lane);
    }
    for (uint32_t n = 16; n > 1u; n >>= 1) {
        __syncthreads();   // the last level's reads of buf are done
        if (warp >= n / 2u && warp < n) {
            buf[warp * 64u + lane] = r0;
            buf[warp * 64u + 32u + lane] = r1;
        }
        __syncthreads();
        if (warp < n / 2u) {
            const uint64_t* b = buf + (warp + n / 2u) * 64u;
            const uint64_t b0 = b[63u - lane], b1 = b[31u - lane];
            r0 = r0 > b0 ? r0 : b0;
            r1 = r1 > b1 ? r1 : b1;
            bitonic_merge64(r0, r1, lane);
        }
    }
    __syncthreads();
    if (warp == 0u) {
        buf[lane] = r0;
        buf[32u + lane] = r1;
    }
    __syncthreads();
}

// How many of a descending 64-key list come before v (ties: list first
// when `or_equal`), by binary search.
__device__ __forceinline__ uint32_t count_before(const uint64_t* list, uint64_t v, bool or_equal) {
    uint32_t lo = 0, hi = kKeep;
    while (lo < hi) {
        const uint32_t mid = (lo + hi) >> 1;
        const bool before = or_equal ? list[mid] >= v : list[mid] > v;
        if (before) lo = mid + 1; else hi = mid;
    }
    return lo;
}

// Merges `lists` descending 64-key lists held in `src` (shared memory)
// pairwise, round by round, each output the pair's top 64 by rank; the
// result is left in src[0..63]. `dst` holds lists/2 + 1 lists.
__device__ void merge_lists(uint64_t* src, uint64_t* dst, uint32_t lists) {
    const uint32_t t = threadIdx.x;
    while (lists > 1) {
        const uint32_t out_lists = (lists + 1u) / 2u;
        for (uint32_t i = t; i < out_lists * 2u * kKeep; i += kSelThreads) {
            const uint32_t pair = i / (2u * kKeep), w = i % (2u * kKeep);
            const uint64_t* A = src + (2u * pair) * kKeep;
            uint64_t* out = dst + pair * kKeep;
            if (2u * pair + 1u >= lists) {   // an odd list out passes through
                if (w < kKeep) out[w] = A[w];
                continue;
            }
            const uint64_t* Bl = A + kKeep;
            uint32_t pos;
            uint64_t v;
            if (w < kKeep) { v = A[w]; pos = w + count_before(Bl, v, false); }
            else { v = Bl[w - kKeep]; pos = (w - kKeep) + count_before(A, v, true); }
            if (pos < kKeep) out[pos] = v;
        }
        __syncthreads();
        for (uint32_t i = t; i < out_lists * kKeep; i += kSelThreads) src[i] = dst[i];
        __syncthreads();
        lists = out_lists;
    }
}

// Takes this CTA's ticket among `of`; true for the last to arrive (which
// resets the ticket for the next step).
__device__ __forceinline__ bool last_to_arrive(unsigned int* ticket, uint32_t of, unsigned int* flag) {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned int seen = atomicAdd(ticket, 1u);
        *flag = seen == of - 1u;
        if (*flag) *ticket = 0u;
    }
    __syncthreads();
    const bool last = *flag != 0u;
    if (last) __threadfence();
    return last;
}

__device__ __forceinline__ uint64_t load_key(const uint32_t* pairs, uint32_t i) {
    const uint32_t bits = __ldcg(pairs + 2u * i), id = __ldcg(pairs + 2u * i + 1u);
    return id == 0xFFFFFFFFu ? 0ull : entry_key(bits, id);
}

__device__ __forceinline__ uint32_t philox_word0(uint32_t c0, uint32_t k0, uint32_t k1) {
    uint32_t c[4] = {c0, 0, 0, 0};
    for (int r = 0; r < 10; ++r) {
        const uint32_t hi0 = __umulhi(0xD2511F53u, c[0]), lo0 = 0xD2511F53u * c[0];
        const uint32_t hi1 = __umulhi(0xCD9E8D57u, c[2]), lo1 = 0xCD9E8D57u * c[2];
        const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
        c[0] = n0; c[1] = lo1; c[2] = n2; c[3] = lo0;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return c[0];
}

// The 64 candidates src[0..63] (descending keys) as (bits, token) pairs to
// `candidates`, then the draw (draw.wgsl:71-163; temperature 0 keeps
// candidate 0, greedy) into the 16-byte record `sampled`. The block's
// threads all call it; row r draws with seed1 + r.
template <typename Args>
__device__ void draw_candidates(const uint64_t* src, const Args& a, uint32_t* candidates, uint32_t* sampled,
                                uint32_t row) {
    const uint32_t t = threadIdx.x;
    // src[0..63]: the candidates, in the reference's order.
    __shared__ uint32_t cand[2 * kKeep];
    __shared__ float weight[kKeep], tempered[kKeep], running[kKeep];
    __shared__ uint32_t above[kKeep];
    __shared__ float total_s;
    if (t < kKeep) {
        entry_pair(src[t], cand + 2u * t);
        candidates[2u * t] = cand[2u * t];
        candidates[2u * t + 1u] = cand[2u * t + 1u];
    }
    __syncthreads();
    // The draw (draw.wgsl:71-163); temperature 0 keeps candidate 0 (greedy).
    const uint32_t k = min(a.top_k ? a.top_k : 1u, kKeep);
    const bool top_p = a.top_p < 1.0f;
    const uint32_t first_bits = cand[0];
    const bool failed = (first_bits & 0x7F800000u) == 0x7F800000u;
    if (t < k) {
        const uint32_t mine_bits = cand[2u * t];
        weight[t] = 0.0f;
        tempered[t] = 0.0f;
        above[t] = 0u;
        if (!failed && mine_bits != 0xFF800000u) {
            const float first = __uint_as_float(first_bits), mine = __uint_as_float(mine_bits);
            if (top_p) weight[t] = exp_nonpositive(mine - first);
            if (a.temperature > 0.0f) tempered[t] = exp_nonpositive((mine - first) / a.temperature);
            above[t] = (a.min_p == 0.0f || mine >= first + a.log_min_p) ? 1u : 0u;
        }
    }
    __syncthreads();
    if (t == 0) {
        const uint32_t pos = a.position ? *a.position : a.position0;
        const uint32_t w0 = philox_word0(pos + a.tokens, a.seed0, a.seed1 + row);
        const float u = static_cast<float>(w0 >> 9) * (1.0f / 8388608.0f) + (1.0f / 16777216.0f);
        if (top_p) {
            float sum = 0.0f;
            for (uint32_t i = 0; i < k; ++i) sum = sum + weight[i];
            if (!failed)
                for (uint32_t i = 0; i < k; ++i) weight[i] = weight[i] / sum;
        }
        uint32_t kept = k;
        float cumulative = 0.0f, tempered_sum = 0.0f;
        for (uint32_t i = 0; i < k; ++i) {
            tempered_sum = tempered_sum + tempered[i];
            running[i] = tempered_sum;
            if (top_p) {
                cumulative = cumulative + weight[i];
                if (cumulative >= a.top_p) { kept = i + 1u; break; }
            }
        }
        uint32_t survivors = 1;
        while (survivors < kept && above[survivors] == 1u) survivors++;
        uint32_t chosen = 0;
        if (a.temperature > 0.0f) {
            const float goal = u * running[survivors - 1u];
            chosen = survivors - 1u;
            for (uint32_t i = 0; i < survivors; ++i)
                if (running[i] > goal) { chosen = i; break; }
        }
        sampled[0] = failed ? 0u : cand[2u * chosen + 1u];
        sampled[1] = failed ? 1u : 0u;
        sampled[2] = __float_as_uint(u);
        sampled[3] = 0u;
    }
}

__global__ void __launch_bounds__(kSelThreads) select_kernel(SelectArgs a) {
    extern __shared__ __align__(16) uint64_t buf[];   // a tile of keys
    __shared__ unsigned int last;
    grid_dependency_wait();
    const uint32_t t = threadIdx.x;
    const uint32_t tile = blockIdx.x;
    // Row blockIdx.y of a batched selection: its own logits, scratch,
    // candidates and record.
    const uint32_t row = blockIdx.y;
    if (row) {
        a.logits += static_cast<size_t>(row) * a.logits_stride;
        a.partials += static_cast<size_t>(row) * gridDim.x * kKeep * 2u;
        a.ticket += static_cast<size_t>(row) * (1u + (gridDim.x + kGroup - 1u) / kGroup);
        a.candidates += static_cast<size_t>(row) * kKeep * 2u;
        a.sampled += static_cast<size_t>(row) * 4u;
    }
    {
        const uint32_t e = tile * kTile + t;
        uint64_t k = 0;
        if (e < a.count) k = entry_key(__float_as_uint(a.logits[e]), e + a.id_offset);
        top_of_tile(k, buf);
    }
    if (t < kKeep) entry_pair(buf[t], a.partials + 2u * (tile * kKeep + t));
    grid_dependents_launch();

    // Level 1: the last tile of each group of kGroup merges the group's
    // lists into the group's first slot. Level 2: the last group merges the
    // groups' lists. Both merge pairwise by rank (merge_lists).
    __shared__ unsigned int flag;
    const uint32_t group = tile / kGroup;
    const uint32_t groups = (gridDim.x + kGroup - 1u) / kGroup;
    const uint32_t in_group = min(kGroup, gridDim.x - group * kGroup);
    if (!last_to_arrive(a.ticket + 1u + group, in_group, &flag)) return;
    uint64_t* work = buf;                   // kGroup lists
    uint64_t* tmp = buf + kGroup * kKeep;   // half as many
    for (uint32_t i = t; i < in_group * kKeep; i += kSelThreads) work[i] = load_key(a.partials, group * kGroup * kKeep + i);
    __syncthreads();
    merge_lists(work, tmp, in_group);
    if (t < kKeep) entry_pair(work[t], a.partials + 2u * (group * kGroup * kKeep + t));
    if (!last_to_arrive(a.ticket, groups, &flag)) return;
    for (uint32_t i = t; i < groups * kKeep; i += kSelThreads)
        work[i] = load_key(a.partials, (i / kKeep) * kGroup * kKeep + i % kKeep);
    __syncthreads();
    merge_lists(work, tmp, groups);
    if (a.candidates_only) {   // a vocabulary shard's top 64, for a merge elsewhere
        if (t < kKeep) entry_pair(work[t], a.candidates + 2u * t);
        return;
    }
    draw_candidates(work, a, a.candidates, a.sampled, row);
}

// Merges `lists` candidate lists of each row (a vocabulary split over ranks:
// list l of row r at ((l·rows + r)·64) pairs) into the row's top 64 — the
// union holds the whole vocabulary's top 64, so these are the candidates of
// one selection over the whole vocabulary — then draws. One CTA a row.
__global__ void __launch_bounds__(kSelThreads) merge_kernel(cb_select_merge a) {
    extern __shared__ __align__(16) uint64_t mbuf[];
    grid_dependency_wait();
    const uint32_t row = blockIdx.x, t = threadIdx.x;
    uint64_t* work = mbuf;
    uint64_t* tmp = mbuf + a.lists * kKeep;
    for (uint32_t i = t; i < a.lists * kKeep; i += kSelThreads)
        work[i] = load_key(a.lists_data, (i / kKeep * a.rows + row) * kKeep + i % kKeep);
    __syncthreads();
    grid_dependents_launch();
    merge_lists(work, tmp, a.lists);
    draw_candidates(work, a, a.candidates + static_cast<size_t>(row) * kKeep * 2u, a.sampled + 4u * row, row);
}

}  // namespace

cudaError_t select_merge_run(const cb_select_merge& a, cudaStream_t stream, bool pdl) {
    if (a.lists == 0 || a.lists > 64 || a.rows == 0) return cudaErrorInvalidValue;
    const size_t smem = (a.lists + a.lists / 2u + 1u) * kKeep * sizeof(uint64_t);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.rows);
    cfg.blockDim = dim3(kSelThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, merge_kernel, a);
}

uint32_t select_tiles(uint32_t count) { return (count + kTile - 1u) / kTile; }

cudaError_t select_run(const SelectArgs& a, cudaStream_t stream, bool pdl) {
    const uint32_t tiles = select_tiles(a.count);
    if (tiles == 0 || tiles > kMaxTiles) return cudaErrorInvalidValue;
    const size_t smem = (kTile > kGroup * kKeep * 3 / 2 ? kTile : kGroup * kKeep * 3 / 2) * sizeof(uint64_t);
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        configured = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(tiles, a.rows > 1 ? a.rows : 1u);
    cfg.blockDim = dim3(kSelThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, select_kernel, a);
}

}  // namespace cb
