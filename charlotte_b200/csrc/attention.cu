// Attention over the f16 KV cache (plainsight-systems/charlotte,
// src/core/kernels/attention/attention.wgsl main :138-360, combine :363-392;
// launcher attention.h:304-320, attention.cpp:27-86).
//
// The reference's arithmetic, per query row at position p and query head h
// (kv head h / G): keys live for p are earliest..p (earliest = p+1-W when
// p+1 > W, else 0). Keys are taken in 64-key chunks fixed by position
// (key_chunks, interface.h:243); within a chunk, in tiles of B = 2048/d keys
// aligned to B, an online softmax in log2 units: the tile's top over its
// live scores, a = 2^(old−top) (1 when equal), e_b = 2^(s_b − top), the
// sum in key order, l = fma(l, a, sum), and O = O·a then O = fma(p_b, v_b, O)
// in key order. s = Σ_w dot(q_w·scale·log2e, k_w) in quads, in order. The
// chunks' (O, m, l) are folded in chunk order with fold_factors/fold_sum/fold
// (:101-127), then O / l. Keys and chunks that are not live contribute
// exactly nothing (a zero weight's product added to a sum that is never −0),
// so they are skipped.
//
// B200 mapping: CTAs a (kv head, tile of rows), at most 16 of them striding
// over the tile's live chunks; each chunk's 64 keys and values staged in
// shared memory once for all its G·rows queries;
// a thread a (query, key) score; a warp a query for the softmax (the tile's
// max and exponentials across lanes, the in-order sums by one lane);
// threads over (query, dimension) for P·V. Every live CTA writes its
// chunk's partial state; the last of the tile's live chunks to finish —
// found by an atomic ticket, no waiting — folds them in order and resets
// the ticket. CTAs of chunks no row reaches (the grid spans the context, so
// a decode graph replays at any position) leave at once. So a decode step is one launch, split over every chunk
// (flash-decoding), and a prefill step the same launch with more row tiles.
#include <cuda_runtime.h>

#include <cstdint>

#include "api_common.h"
#include "kernels.h"
#include "numerics.cuh"
#include "rope_math.cuh"
#include "tma.cuh"

namespace cb {

namespace {

constexpr uint32_t kChunk = 64;
constexpr uint32_t kAttnThreads = 256;
constexpr uint32_t kMaxQueries = 16;   // queries (rows × G) a CTA works
// Halves past a staged key or value row's d: a 16-byte pad, so the rows of
// consecutive keys (read by consecutive lanes) start on different banks.
constexpr uint32_t kRowPad = 8;
constexpr uint32_t kChunkSlots = 16;   // CTAs a (kv head, row tile) takes, striding over its live chunks

struct Geometry {
    uint32_t rows_per_tile;   // query rows a CTA takes
    uint32_t G;               // query heads a kv head
};

// Batched decode (rows are sequences): a row a tile, each over its own cache.
__host__ __device__ inline Geometry geometry_of(uint32_t query_heads, uint32_t kv_heads, bool sequences) {
    Geometry g;
    g.G = query_heads / kv_heads;
    g.rows_per_tile = sequences ? 1u : (kMaxQueries / g.G > 0 ? kMaxQueries / g.G : 1);
    return g;
}

__host__ __device__ inline size_t attention_smem(uint32_t d, uint32_t queries) {
    return 2ull * kChunk * (d + kRowPad) * 2u   // K and V, f16, padded rows
           + static_cast<size_t>(queries) * d * 4u   // q·scale·log2e
           + static_cast<size_t>(queries) * kChunk * 4u   // scores, then weights
           + static_cast<size_t>(queries) * 8u * 4u       // a tile's alpha (≤ 8 tiles)
           + static_cast<size_t>(queries) * 4u * 4u       // m, l, live, spare
           + static_cast<size_t>(queries) * 16u * 4u;     // each tile's top and sum
}

// Cluster fold (decode shapes: a row a tile, Q = G queries): the floats of
// rank 0's shared memory that take every chunk's partial and (m, l), after
// the layout above.
__host__ __device__ inline size_t cluster_fold_floats(uint32_t d, uint32_t G) {
    return static_cast<size_t>(kChunkSlots) * G * (d + 2u);
}

__device__ __forceinline__ uint32_t earliest_of(uint32_t p, uint32_t window) {
    return p + 1u > window ? p + 1u - window : 0u;
}


// Stages keys and values j_lo..j_hi-1 (absolute positions) of the chunk at
// key0 into its shared tiles: every thread of the CTA copies 16-byte pieces
// of the rows (asynchronous copies through L2, consecutive threads along a
// row). With `arrive`, each thread then arrives on `bar` once its copies so
// far have landed (the barrier counts one arrival a thread); without, the
// copies join the phase whose arrivals come with a later batch. (One bulk
// copy a row was measured at ~3.7 us to issue a chunk's 128 rows: the rows
// are small and the copy unit takes them one at a time.)
__device__ __forceinline__ void stage_keys(const AttentionArgs& a, const uint16_t* kc, const uint16_t* vc, uint16_t* ks,
                                           uint16_t* vs, uint32_t key0, uint32_t j_lo, uint32_t j_hi, uint32_t kvh,
                                           uint32_t d, uint64_t* bar, bool arrive) {
    const uint32_t n = j_hi > j_lo ? j_hi - j_lo : 0u;
    const uint32_t per_row = d / 8u;   // 16-byte pieces a row
    const uint32_t pieces = 2u * n * per_row;
    const uint32_t slot0 = key0 % a.slots;   // the ring's slot of the chunk's first key
    for (uint32_t i = threadIdx.x; i < pieces; i += kAttnThreads) {
        const uint32_t row = i / per_row, w = i % per_row;
        const bool value = row >= n;
        const uint32_t b = j_lo - key0 + (value ? row - n : row);
        uint32_t slot = slot0 + b;
        while (slot >= a.slots) slot -= a.slots;
        const size_t at = (static_cast<size_t>(slot) * a.kv_heads + kvh) * d + 8u * w;
        cp_async16((value ? vs : ks) + b * (d + kRowPad) + 8u * w, (value ? vc : kc) + at);
    }
    if (arrive) cp_async_mbar_arrive(bar);
}

// The chunks' fold in chunk order (fold_factors/fold_sum/fold,
// attention.wgsl:101-127): for each live chunk c of a query, with top the
// largest of the earlier chunks' tops, (fa, fb) = (0, 1) for the first,
// (1, 1) when top = m_c, (1, 2^(m_c − top)) when top > m_c, else
// (2^(top − m_c), 1); then l = fma(l, fa, l_c·fb) and o = fma(o, fa,
// o_c·fb). The factors depend on the partials only through that running
// top, a prefix maximum, so here a warp a query finds every chunk's
// (fa, fb) of a block of 32 chunks at once (a scan of maxima across lanes,
// then each lane's exp2), and then every (query, dimension) runs its o and
// l chains in chunk order — the same operations on the same operands as one
// chunk after the other, so the same bits.
// `stat_of(c, m, &cm, &cl)` gives chunk c's (m, l) for query m,
// `part_of(c, m, e)` its partial; queries' chunk ranges from
// `range_of(m, &c0, &c1)`; `write(m, e, o / l)` takes each output. `fac`
// holds Q·64 floats of scratch, `lfac` Q·32; the CTA must have met a
// barrier since their last readers.
template <uint32_t D, typename Range, typename Stat, typename Part, typename Write>
__device__ __forceinline__ void fold_chunks(uint32_t Q, float* fac, float* lfac, Range range_of, Stat stat_of,
                                            Part part_of, Write write, uint32_t lane, uint32_t wid) {
    uint32_t lo = 0xFFFFFFFFu, hi = 0;
    for (uint32_t m = 0; m < Q; ++m) {
        uint32_t c0, c1;
        range_of(m, &c0, &c1);
        lo = min(lo, c0);
        hi = max(hi, c1);
    }
    constexpr uint32_t warps = kAttnThreads / 32u;
    // Every chunk's (fa, fb) of a block of 32 chunks, a warp a query.
    float carry[kMaxQueries / warps];   // the running top of each of this warp's queries
#pragma unroll
    for (uint32_t k = 0; k < kMaxQueries / warps; ++k) carry[k] = -INFINITY;
    auto factors = [&](uint32_t base) {
#pragma unroll
        for (uint32_t k = 0; k < kMaxQueries / warps; ++k) {
            const uint32_t m = wid + k * warps;
            if (m >= Q) break;
            uint32_t c0, c1;
            range_of(m, &c0, &c1);
            const uint32_t c = base + lane;
            const bool in = c >= c0 && c <= c1;
            float cm = -INFINITY, cl = 0.0f;
            if (in) stat_of(c, m, &cm, &cl);
            float incl = cm;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const float v = __shfl_up_sync(0xFFFFFFFFu, incl, off);
                if (lane >= static_cast<uint32_t>(off)) incl = fmaxf(incl, v);
            }
            const float before = __shfl_up_sync(0xFFFFFFFFu, incl, 1);
            const float top = fmaxf(carry[k], lane ? before : -INFINITY);   // the running top before c
            float fa = 1.0f, fb = 1.0f;
            if (in) {
                if (c == c0) { fa = 0.0f; fb = 1.0f; }
                else if (top == cm) { fa = 1.0f; fb = 1.0f; }
                else if (top > cm) { fa = 1.0f; fb = exp2_np(cm - top); }
                else { fa = exp2_np(top - cm); fb = 1.0f; }
            }
            fac[(m * 32u + lane) * 2u] = fa;
            fac[(m * 32u + lane) * 2u + 1u] = fb;
            lfac[m * 32u + lane] = cl * fb;
            carry[k] = fmaxf(carry[k], __shfl_sync(0xFFFFFFFFu, incl, 31));
        }
    };
    // One output's chains over the block's chunks [c0, c1], its partials
    // loaded 16 at a time before their fmas.
    auto chain = [&](uint32_t base, uint32_t m, uint32_t e, uint32_t c0, uint32_t c1, float& o, float& l) {
#pragma unroll 1
        for (uint32_t c = c0; c <= c1; c += 16u) {
            float co[16];
#pragma unroll
            for (uint32_t k = 0; k < 16u; ++k) co[k] = c + k <= c1 ? part_of(c + k, m, e) : 0.0f;
#pragma unroll
            for (uint32_t k = 0; k < 16u; ++k)
                if (c + k <= c1) {
                    const uint32_t f = m * 32u + (c + k - base);
                    const float fa = fac[2u * f];
                    o = fmaf(o, fa, co[k] * fac[2u * f + 1u]);
                    l = fmaf(l, fa, lfac[f]);
                }
        }
    };
    if (hi - lo < 32u) {
        // One block (up to 2,048 keys): its factors once, then the outputs
        // in groups of the CTA's threads.
        factors(lo);
        __syncthreads();
        // A thread's outputs (threadIdx.x + 256·j) share the dimension e
        // (the CTA's threads are a whole number of D). With more than one,
        // four at a time run their chains together, chunk by chunk in order,
        // each over its own query's chunks, four chunks' partials of each
        // loaded before their fmas — the operations of `chain`, interleaved.
        static_assert(kAttnThreads % D == 0, "a thread's outputs share one dimension");
        constexpr uint32_t kStep = kAttnThreads / D;   // queries between a thread's outputs
        if (Q <= kStep) {
            const uint32_t m = threadIdx.x / D, e = threadIdx.x % D;
            if (m < Q) {
                uint32_t c0, c1;
                range_of(m, &c0, &c1);
                float o = 0.0f, l = 0.0f;
                chain(lo, m, e, c0, c1, o, l);
                write(m, e, o / l);
            }
            return;
        }
        const uint32_t e = threadIdx.x % D;
#pragma unroll 1
        for (uint32_t mb = threadIdx.x / D; mb < Q; mb += 4u * kStep) {
            uint32_t c0[4], c1[4];
            float o[4], l[4];
#pragma unroll
            for (uint32_t j = 0; j < 4u; ++j) {
                c0[j] = 1u;
                c1[j] = 0u;   // no chunks: past the CTA's queries
                if (mb + j * kStep < Q) range_of(mb + j * kStep, &c0[j], &c1[j]);
                o[j] = 0.0f;
                l[j] = 0.0f;
            }
#pragma unroll 1
            for (uint32_t c = lo; c <= hi; c += 4u) {
                float co[4][4];
#pragma unroll
                for (uint32_t j = 0; j < 4u; ++j)
#pragma unroll
                    for (uint32_t k = 0; k < 4u; ++k) {
                        const uint32_t cc = c + k;
                        co[j][k] = cc >= c0[j] && cc <= c1[j] ? part_of(cc, mb + j * kStep, e) : 0.0f;
                    }
#pragma unroll
                for (uint32_t k = 0; k < 4u; ++k)
#pragma unroll
                    for (uint32_t j = 0; j < 4u; ++j) {
                        const uint32_t cc = c + k;
                        if (cc >= c0[j] && cc <= c1[j]) {
                            const uint32_t f = (mb + j * kStep) * 32u + (cc - lo);
                            const float fa = fac[2u * f];
                            o[j] = fmaf(o[j], fa, co[j][k] * fac[2u * f + 1u]);
                            l[j] = fmaf(l[j], fa, lfac[f]);
                        }
                    }
            }
#pragma unroll
            for (uint32_t j = 0; j < 4u; ++j)
                if (mb + j * kStep < Q) write(mb + j * kStep, e, o[j] / l[j]);
        }
        return;
    }
    // Longer: the outputs in groups of the CTA's threads, each group
    // walking the blocks (their factors again for each group).
    for (uint32_t i0 = 0; i0 < Q * D; i0 += kAttnThreads) {
        if (i0) {
            __syncthreads();   // the last group's reads of the factors are done
#pragma unroll
            for (uint32_t k = 0; k < kMaxQueries / warps; ++k) carry[k] = -INFINITY;
        }
        const uint32_t i = i0 + threadIdx.x;
        const uint32_t m = i / D, e = i % D;
        uint32_t mc0 = 0, mc1 = 0;
        if (i < Q * D) range_of(m, &mc0, &mc1);
        float o = 0.0f, l = 0.0f;
        for (uint32_t base = lo; base <= hi; base += 32u) {
            factors(base);
            __syncthreads();
            if (i < Q * D && mc1 >= base && mc0 <= base + 31u)
                chain(base, m, e, max(mc0, base), min(mc1, base + 31u), o, l);
            if (base + 32u <= hi) __syncthreads();   // before the next block's factors
        }
        if (i < Q * D) write(m, e, o / l);
    }
}

// The step's rope done in the prologue (decode shapes, `fused`): r is that
// rope step's arguments.
template <uint32_t D>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(AttentionArgs a, RopeArgs r, uint32_t fused,
                                                                 unsigned int* fault) {
    extern __shared__ __align__(16) uint8_t smem[];
    constexpr uint32_t d = D;
    constexpr uint32_t B = 2048u / D;           // a tile's keys
    constexpr uint32_t tiles = kChunk / B;
    const bool seqs = a.rows_are_sequences != 0;
    const Geometry geo = geometry_of(a.query_heads, a.kv_heads, seqs);
    const uint32_t G = geo.G;
    const uint32_t kvh = blockIdx.x;
    const uint32_t rt = blockIdx.z;
    const uint32_t spin = spin_limit_of(fault);   // read early: off the first wait's path
    // Batched decode: this tile's one row is its sequence's, over its cache.
    const size_t cache_at = seqs ? static_cast<size_t>(rt) * a.sequence_stride : 0u;
    const uint16_t* kc = a.key_cache + cache_at;
    const uint16_t* vc = a.value_cache + cache_at;
    // The step's position was written before the launches preceding this one
    // (by the host, or by the last step's closing launch), so it is read
    // before the dependency wait, as are the keys of earlier steps.
    const uint32_t pos0 = a.position ? *a.position : a.position0;
    // The fused rope's turn (and llama3 factor) of this thread's angle (d/2
    // angles, one a thread), loaded beside the position so the two loads
    // share one round trip.
    static_assert(D / 2u <= kAttnThreads, "one angle a thread");
    const bool angle_thread = fused && threadIdx.x < D / 2u;
    const float turn_k = angle_thread ? __ldg(r.turns + threadIdx.x) : 0.0f;
    const float factor_k = angle_thread && r.factors ? __ldg(r.factors + threadIdx.x) : 1.0f;
    const uint32_t row0 = rt * geo.rows_per_tile;
    const uint32_t rows = min(geo.rows_per_tile, a.tokens - row0);
    const uint32_t Q = rows * G;
    const uint32_t lane = threadIdx.x & 31u, wid = threadIdx.x >> 5;

    const uint32_t pitch = d + kRowPad;   // halves a staged key or value row takes
    uint16_t* ks = reinterpret_cast<uint16_t*>(smem);
    uint16_t* vs = ks + kChunk * pitch;
    float* qs = reinterpret_cast<float*>(vs + kChunk * pitch);
    float* ps = qs + kMaxQueries * d;                 // [Q][64]
    float* alpha = ps + kMaxQueries * kChunk;         // [Q][8]
    float* stat = alpha + kMaxQueries * 8u;           // [Q][4]: m, l
    float* tops = stat + kMaxQueries * 4u;            // [Q][8]: each tile's top (-inf: no live key)
    float* sums = tops + kMaxQueries * 8u;            // [Q][8]: each tile's sum of weights
    float* fold_part = sums + kMaxQueries * 8u;       // cluster fold, rank 0: [slot][Q][d], then [slot][Q][2]
    float* fold_stat = fold_part + kChunkSlots * G * d;

    // The tile's live chunks: every chunk some row's keys reach.
    const uint32_t p_first = pos0 + (seqs ? 0u : row0), p_last = p_first + (seqs ? 0u : rows - 1u);
    const uint32_t live_first = earliest_of(p_first, a.window) / kChunk;
    const uint32_t live_chunks = p_last / kChunk - live_first + 1u;
    // Cluster fold: the tile's chunk CTAs are one cluster (the launch makes
    // them one for decode shapes when it fits) and each has at most one
    // live chunk. Each CTA then stores its partial and (m, l) into rank 0's
    // shared memory; after one cluster barrier, which every CTA of the
    // cluster meets, chunk or not, rank 0 folds them. Otherwise partials go
    // through global memory and the last CTA to take a ticket folds them.
    const bool cluster_fold = cluster_size() > 1u && live_chunks <= gridDim.y;
    if (blockIdx.y >= live_chunks && !cluster_fold) {   // no chunk for this slot: no ticket either
        grid_dependency_wait();
        return;
    }
    // One mbarrier phase a chunk for its keys and values.
    __shared__ uint64_t kv_bar;
    uint32_t kv_phase = 0;
    if (threadIdx.x == 0) {
        mbar_init(&kv_bar, kAttnThreads);   // a thread's arrival once its copies of the phase land
        fence_barrier_init();
    }
    __syncthreads();
    // This slot's first chunk's keys of earlier steps (below pos0), in flight
    // while the launch before this one finishes.
    const uint32_t c_first = live_first + blockIdx.y;
    {
        const uint32_t key0 = c_first * kChunk;
        const uint32_t j_hi = min(key0 + kChunk, max(pos0, key0));
        stage_keys(a, kc, vc, ks, vs, key0, key0, j_hi, kvh, d, &kv_bar, false);
    }
    const bool working = blockIdx.y < live_chunks;
    // The fused rope's angle table for the rows' position (decode shapes: one
    // position a tile), into the score buffer, free until the scores.
    float* cosines = ps;
    float* sines = ps + d / 2u;
    if (working && angle_thread)
        rope_angle(p_first, turn_k, factor_k, r.factors != nullptr, &cosines[threadIdx.x], &sines[threadIdx.x]);
    grid_dependency_wait();

    // The fused rope: G query heads (and, in the CTA whose chunks hold the
    // newest key, that key and its value), d/8 threads a head as in the rope
    // launch. Queries go to the q stage scaled as below; the key and value,
    // packed f16, to the caches and — when the newest key's chunk is this
    // CTA's first — straight into the chunk's stage.
    if (fused && working) {
        __syncthreads();   // the angle table
        const uint32_t lanes = d / 8u;
        const uint32_t newest_chunk = p_first / kChunk;
        const bool newest = (newest_chunk - live_first) % gridDim.y == blockIdx.y;
        const uint32_t heads = G + (newest ? 2u : 0u);
        if (threadIdx.x < (heads * lanes + 31u) / 32u * 32u) {
            const uint32_t head = threadIdx.x / lanes, lane = threadIdx.x % lanes;
            const bool valid = head < heads, is_query = head < G, is_value = head == G + 1u;
            const size_t row = row0;
            const float* src = is_query ? r.query + (row * a.query_heads + kvh * G + head) * d
                                        : (is_value ? r.value : r.key) + (row * a.kv_heads + kvh) * d;
            float4 x0 = valid ? reinterpret_cast<const float4*>(src)[lane] : make_float4(0.f, 0.f, 0.f, 0.f);
            float4 x1 = valid ? reinterpret_cast<const float4*>(src)[lane + lanes] : make_float4(0.f, 0.f, 0.f, 0.f);
            rope_head(x0, x1, lane, lanes, d, r.query_gain != nullptr, r.epsilon, is_query ? r.query_gain : r.key_gain,
                      !is_value, r.halves != 0, cosines, sines);
            if (valid && is_query) {
                float4* q4 = reinterpret_cast<float4*>(qs + head * d);
                q4[lane] = make_float4(x0.x * a.scale_log2e, x0.y * a.scale_log2e, x0.z * a.scale_log2e,
                                       x0.w * a.scale_log2e);
                q4[lane + lanes] = make_float4(x1.x * a.scale_log2e, x1.y * a.scale_log2e, x1.z * a.scale_log2e,
                                               x1.w * a.scale_log2e);
            } else if (valid) {
                uint16_t* cache = (is_value ? r.value_cache : r.key_cache) + (seqs ? row * r.sequence_stride : 0u);
                uint16_t* dst = cache + (static_cast<size_t>(p_first % a.slots) * a.kv_heads + kvh) * d;
                store_f16x4(dst + 4u * lane, x0);
                store_f16x4(dst + 4u * (lane + lanes), x1);
                if (newest_chunk == c_first) {
                    uint16_t* st = (is_value ? vs : ks) + (p_first - c_first * kChunk) * pitch;
                    store_f16x4(st + 4u * lane, x0);
                    store_f16x4(st + 4u * (lane + lanes), x1);
                }
            }
        }
        // The new rows' global stores before a bulk copy that reads them (a
        // later chunk of this CTA's), and the angle table's last reads.
        fence_proxy_async_global();
        __syncthreads();
    }

    // Queries m = r·G + g: row r, head kvh·G + g, scaled into log2 units.
    for (uint32_t i = threadIdx.x; i < (working && !fused ? Q * d : 0u); i += kAttnThreads) {
        const uint32_t m = i / d, e = i % d;
        const uint32_t r = m / G, h = kvh * G + m % G;
        qs[m * d + e] = a.query[(static_cast<size_t>(row0 + r) * a.query_heads + h) * d + e] * a.scale_log2e;
    }
    bool failed = false;
    for (uint32_t c = c_first; c <= p_last / kChunk; c += gridDim.y) {
        const uint32_t key0 = c * kChunk;
        const bool first_chunk = c == c_first;
        if (!first_chunk) {
            __syncthreads();      // the last chunk's reads of ks, vs, ps are done
            fence_proxy_async();  // and ordered before the copy engine's writes
        }
        // The chunk's keys this step wrote (for later chunks, all of them);
        // positions past p_last are never live and are not staged. A fused
        // rope's newest key, when this is its chunk and the CTA's first, is
        // staged already.
        {
            const uint32_t j_lo = first_chunk ? max(key0, min(pos0, key0 + kChunk)) : key0;
            const bool staged_new = fused && first_chunk && p_last / kChunk == c;
            const uint32_t j_hi = min(key0 + kChunk, staged_new ? p_last : p_last + 1u);
            stage_keys(a, kc, vc, ks, vs, key0, j_lo, max(j_lo, j_hi), kvh, d, &kv_bar, true);
        }
        if (!__syncthreads_and(mbar_wait(&kv_bar, kv_phase, fault, spin))) {
            // A copy did not land in time (the fault word is set; the whole
            // CTA agrees): wait once more, bounded, so none is left writing
            // this CTA's shared memory, and stop (the step reports failure).
            mbar_wait(&kv_bar, kv_phase, nullptr);
            failed = true;
            break;
        }
        kv_phase ^= 1u;
        // Scores: s = Σ_w dot(q_w, k_w) in quads, in order.
        for (uint32_t i = threadIdx.x; i < Q * kChunk; i += kAttnThreads) {
            const uint32_t m = i / kChunk, b = i % kChunk;
            const uint32_t p = p_first + (seqs ? 0u : m / G);
            const uint32_t j = key0 + b;
            float s = 0.0f;
            if (j <= p && j >= earliest_of(p, a.window)) {
                // Two quads a 16-byte read of the key row (padded rows:
                // consecutive lanes' keys on distinct banks).
                const float4* q4 = reinterpret_cast<const float4*>(qs + m * d);
                const uint4* k8 = reinterpret_cast<const uint4*>(ks + b * pitch);
#pragma unroll 4
                for (uint32_t w = 0; w < d / 8u; ++w) {
                    const uint4 kw = k8[w];
                    const float4 ka = make_float4(fp16_bits_to_f32(kw.x & 0xFFFF), fp16_bits_to_f32(kw.x >> 16),
                                                  fp16_bits_to_f32(kw.y & 0xFFFF), fp16_bits_to_f32(kw.y >> 16));
                    const float4 kb = make_float4(fp16_bits_to_f32(kw.z & 0xFFFF), fp16_bits_to_f32(kw.z >> 16),
                                                  fp16_bits_to_f32(kw.w & 0xFFFF), fp16_bits_to_f32(kw.w >> 16));
                    s = s + dot4(q4[2u * w], ka);
                    s = s + dot4(q4[2u * w + 1u], kb);
                }
            }
            ps[m * kChunk + b] = s;
        }
        __syncthreads();
        // The online softmax, tile by tile in key order, a warp a (query,
        // tile): the tile's top (a max: any order gives its bits); then,
        // with the running top before the tile (the tops of the earlier
        // tiles, in order), old, top = max(old, tile top), a = 2^(old − top)
        // (1 when equal), each live key's 2^(s − top) and the tile's sum
        // from zero in key order; then, a thread a query, l = fma(l, a,
        // sum) over the tiles with live keys, in order.
        {
            // A warp takes 32/B (query, tile) pairs at once, B lanes each
            // (one a key); the shuffles stay within a pair's lanes.
            const uint32_t pairs = Q * tiles;
            constexpr uint32_t kPairs = 32u / B;
            const uint32_t seg = lane / B, sl = lane % B;
            for (uint32_t w0 = wid * kPairs; w0 < pairs; w0 += (kAttnThreads / 32u) * kPairs) {
                const uint32_t w = w0 + seg;
                const uint32_t m = w < pairs ? w / tiles : 0u, t = w < pairs ? w % tiles : 0u;
                const uint32_t p = p_first + (seqs ? 0u : m / G);
                const uint32_t j = key0 + t * B + sl;
                const bool live = w < pairs && j <= p && j >= earliest_of(p, a.window);
                float top = live ? ps[m * kChunk + t * B + sl] : -INFINITY;
#pragma unroll
                for (uint32_t o = B / 2u; o > 0; o >>= 1) top = fmaxf(top, __shfl_xor_sync(0xFFFFFFFFu, top, o, B));
                if (sl == 0 && w < pairs) tops[m * 8u + t] = top;
            }
            __syncthreads();
            for (uint32_t w0 = wid * kPairs; w0 < pairs; w0 += (kAttnThreads / 32u) * kPairs) {
                const uint32_t w = w0 + seg;
                const uint32_t m = w < pairs ? w / tiles : 0u, t = w < pairs ? w % tiles : 0u;
                const uint32_t p = p_first + (seqs ? 0u : m / G);
                const uint32_t j = key0 + t * B + sl;
                const bool live = w < pairs && j <= p && j >= earliest_of(p, a.window);
                bool chunk_live = false;
                float chunk_m = 0.0f, al = 1.0f;
#pragma unroll
                for (uint32_t u = 0; u < tiles; ++u) {
                    const float tt = tops[m * 8u + u];
                    if (u > t || tt == -INFINITY) continue;   // past tile t, or no live key in tile u
                    const float old = chunk_live ? chunk_m : tt;
                    const float top = fmaxf(old, tt);
                    if (u == t) al = old == top ? 1.0f : exp2_np(old - top);
                    chunk_m = top;
                    chunk_live = true;
                }
                const float e = live ? exp2_np(ps[m * kChunk + t * B + sl] - chunk_m) : 0.0f;
                __syncwarp();
                if (w < pairs) ps[m * kChunk + t * B + sl] = e;
                float sum = 0.0f;   // in key order
#pragma unroll
                for (uint32_t b = 0; b < B; ++b) sum = sum + __shfl_sync(0xFFFFFFFFu, e, b, B);
                if (sl == 0 && w < pairs) {
                    alpha[m * 8u + t] = al;
                    sums[m * 8u + t] = sum;
                }
            }
            __syncthreads();
            for (uint32_t m = threadIdx.x; m < Q; m += kAttnThreads) {
                bool chunk_live = false;
                float chunk_m = 0.0f, chunk_l = 0.0f;
#pragma unroll
                for (uint32_t u = 0; u < tiles; ++u) {
                    const float tt = tops[m * 8u + u];
                    if (tt == -INFINITY) continue;
                    const float old = chunk_live ? chunk_m : tt;
                    chunk_m = fmaxf(old, tt);
                    chunk_l = fmaf(chunk_l, alpha[m * 8u + u], sums[m * 8u + u]);
                    chunk_live = true;
                }
                stat[m * 4u + 0] = chunk_m;
                stat[m * 4u + 1] = chunk_live ? chunk_l : 0.0f;
            }
        }
        __syncthreads();
        // O = O·a_t, then fma(p_b, v_b, O) in key order; the chunk's partial.
        // A key of weight 0 (not live for this query) adds exactly nothing —
        // fma(0, v, o) = o for the finite values the cache holds — so the
        // loop needs no test; keys past p_last, never staged, are left out.
        const uint32_t valid = min(kChunk, p_last + 1u - key0);
        // Output (m, e) into rank 0's slot for this CTA's chunk (slot =
        // rank), or to the partials in global memory.
        auto put = [&](uint32_t m, uint32_t e, float o) {
            if (cluster_fold) {
                const uint32_t slot = blockIdx.y;
                st_cluster_f32(cluster_map(fold_part + (slot * G + m) * d + e, 0u), o);
                if (e == 0) {
                    st_cluster_f32(cluster_map(fold_stat + (slot * G + m) * 2u, 0u), stat[m * 4u]);
                    st_cluster_f32(cluster_map(fold_stat + (slot * G + m) * 2u + 1u, 0u), stat[m * 4u + 1u]);
                }
            } else {
                const uint32_t r = m / G, h = kvh * G + m % G;
                const size_t at = (static_cast<size_t>(c) * a.tokens + row0 + r) * a.query_heads + h;
                a.partials[at * d + e] = o;
                if (e == 0) {
                    a.stats[at * 2u] = stat[m * 4u];
                    a.stats[at * 2u + 1u] = stat[m * 4u + 1u];
                }
            }
        };
        if (Q * d <= kAttnThreads) {
            // One output a thread.
            const uint32_t m = threadIdx.x / d, e = threadIdx.x % d;
            if (m < Q) {
                float o = 0.0f;
                // Eight keys at a time (every tile is a whole number of
                // eights): at a tile's first key O·a_t, then the keys' fmas
                // in key order — their weights (two 16-byte reads) and values
                // loaded first, unconditionally (every row of the stage is in
                // bounds), keys from `valid` on (never staged) skipped.
#pragma unroll 2
                for (uint32_t b0 = 0; b0 < kChunk; b0 += 8u) {
                    const float4* p4 = reinterpret_cast<const float4*>(ps + m * kChunk + b0);
                    const float4 pa = p4[0], pb = p4[1];
                    const float pw[8] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
                    float vv[8];
#pragma unroll
                    for (int k = 0; k < 8; ++k) vv[k] = fp16_bits_to_f32(vs[(b0 + k) * pitch + e]);
                    if (b0 % B == 0) o = o * alpha[m * 8u + b0 / B];
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                        if (b0 + k < valid) o = fmaf(pw[k], vv[k], o);
                }
                put(m, e, o);
            }
        } else {
            // A thread's outputs share the dimension e (the CTA's threads are
            // a whole number of d): four at a time, each value loaded once
            // for all four, their chains — independent — advancing together.
            constexpr uint32_t kStep = kAttnThreads / D;
            const uint32_t e = threadIdx.x % d;
#pragma unroll 1
            for (uint32_t mb = threadIdx.x / d; mb < Q; mb += 4u * kStep) {
                float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 2
                for (uint32_t b0 = 0; b0 < kChunk; b0 += 8u) {
                    float vv[8];
#pragma unroll
                    for (int k = 0; k < 8; ++k) vv[k] = fp16_bits_to_f32(vs[(b0 + k) * pitch + e]);
#pragma unroll
                    for (uint32_t j = 0; j < 4u; ++j) {
                        // Queries past the CTA's last read its row (results discarded).
                        const uint32_t m = min(mb + j * kStep, Q - 1u);
                        const float4* p4 = reinterpret_cast<const float4*>(ps + m * kChunk + b0);
                        const float4 pa = p4[0], pb = p4[1];
                        const float pw[8] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
                        if (b0 % B == 0) o[j] = o[j] * alpha[m * 8u + b0 / B];
#pragma unroll
                        for (int k = 0; k < 8; ++k)
                            if (b0 + k < valid) o[j] = fmaf(pw[k], vv[k], o[j]);
                    }
                }
#pragma unroll
                for (uint32_t j = 0; j < 4u; ++j)
                    if (mb + j * kStep < Q) put(mb + j * kStep, e, o[j]);
            }
        }
    }
    grid_dependents_launch();

    if (cluster_fold) {
        cluster_sync();   // every chunk's partial and (m, l) is in rank 0's shared memory
        if (cluster_rank() != 0u) return;
        // The chunks (slot = chunk − the tile's first live chunk) folded in
        // chunk order.
        fold_chunks<D>(
            Q, ps, qs, [&](uint32_t m, uint32_t* c0, uint32_t* c1) {
                const uint32_t p = p_first + (seqs ? 0u : m / G);
                *c0 = earliest_of(p, a.window) / kChunk;
                *c1 = p / kChunk;
            },
            [&](uint32_t c, uint32_t m, float* cm, float* cl) {
                const uint32_t slot = c - live_first;
                *cm = fold_stat[(slot * G + m) * 2u];
                *cl = fold_stat[(slot * G + m) * 2u + 1u];
            },
            [&](uint32_t c, uint32_t m, uint32_t e) { return fold_part[((c - live_first) * G + m) * d + e]; },
            [&](uint32_t m, uint32_t e, float v) {
                a.out[(static_cast<size_t>(row0 + m / G) * a.query_heads + kvh * G + m % G) * d + e] = v;
            },
            lane, wid);
        return;
    }
    if (failed) return;   // without a ticket: the step reports failure

    // The last of the tile's chunk CTAs to finish folds the chunks in order.
    __shared__ unsigned int last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned int* ticket = a.tickets + rt * a.kv_heads + kvh;
        const unsigned int seen = atomicAdd(ticket, 1u);
        last = seen == min(gridDim.y, live_chunks) - 1u;
        if (last) *ticket = 0u;   // ready for the next step
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    // The chunks' partials (global memory, through L2) folded in chunk order.
    auto at_of = [&](uint32_t c, uint32_t m) {
        return (static_cast<size_t>(c) * a.tokens + row0 + m / G) * a.query_heads + kvh * G + m % G;
    };
    fold_chunks<D>(
        Q, ps, qs, [&](uint32_t m, uint32_t* c0, uint32_t* c1) {
            const uint32_t p = p_first + (seqs ? 0u : m / G);
            *c0 = earliest_of(p, a.window) / kChunk;
            *c1 = p / kChunk;
        },
        [&](uint32_t c, uint32_t m, float* cm, float* cl) {
            const size_t at = at_of(c, m);
            *cm = __ldcg(a.stats + at * 2u);
            *cl = __ldcg(a.stats + at * 2u + 1u);
        },
        [&](uint32_t c, uint32_t m, uint32_t e) { return __ldcg(a.partials + at_of(c, m) * d + e); },
        [&](uint32_t m, uint32_t e, float v) {
            a.out[(static_cast<size_t>(row0 + m / G) * a.query_heads + kvh * G + m % G) * d + e] = v;
        },
        lane, wid);
}

}  // namespace

uint32_t attention_row_tiles(uint32_t tokens, uint32_t query_heads, uint32_t kv_heads, bool sequences) {
    const Geometry g = geometry_of(query_heads, kv_heads, sequences);
    return (tokens + g.rows_per_tile - 1) / g.rows_per_tile;
}

namespace {

template <uint32_t D>
cudaError_t launch_attention(const AttentionArgs& a, cudaStream_t stream, bool pdl, size_t base_smem,
                             size_t cluster_smem, bool decode_shape, uint32_t slots) {
    auto kernel = attention_kernel<D>;
    const Geometry geo = geometry_of(a.query_heads, a.kv_heads, a.rows_are_sequences != 0);
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.kv_heads, slots, (a.tokens + geo.rows_per_tile - 1) / geo.rows_per_tile);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    // A (kv head, row tile)'s chunk CTAs as one cluster, when every one of
    // the launch's clusters can be resident at once at this shared-memory
    // size (the occupancy calculator asked once a cluster size): clusters
    // past that would wait for a whole cluster to finish, doubling the
    // launch (measured: 8 clusters of 16 CTAs at head dimension 256, one
    // of them a second wave).
    static int cluster_room[kChunkSlots + 1] = {};   // 0 unknown, else 1 + the clusters resident at once
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = slots;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    const bool can_cluster = decode_shape && slots > 1 && cluster_smem <= 200u * 1024u;
    if (can_cluster && cluster_room[slots] == 0) {
        cfg.numAttrs = 2;
        cfg.dynamicSmemBytes = cluster_smem;
        int clusters = 0;
        const cudaError_t e = cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg);   // any arguments
        if (e != cudaSuccess) cudaGetLastError();
        cluster_room[slots] = 1 + (e == cudaSuccess && clusters > 0 ? clusters : 0);
    }
    const uint64_t clusters_needed = static_cast<uint64_t>(cfg.gridDim.x) * cfg.gridDim.z;
    const bool cluster = can_cluster && static_cast<uint64_t>(cluster_room[slots] - 1) >= clusters_needed;
    cfg.numAttrs = cluster ? 2 : 1;
    cfg.dynamicSmemBytes = cluster ? cluster_smem : base_smem;
    RopeArgs r{};
    if (a.rope) r = *a.rope;
    return cudaLaunchKernelEx(&cfg, kernel, a, r, a.rope ? 1u : 0u, fault_word());
}

}  // namespace

cudaError_t attention_run(const AttentionArgs& a, cudaStream_t stream, bool pdl) {
    if (!a.rows_are_sequences && a.tokens >= kPrefillAttentionRows && attention_prefill_fits(a))
        return attention_prefill_run(a, stream, pdl);
    const Geometry geo = geometry_of(a.query_heads, a.kv_heads, a.rows_are_sequences != 0);
    if (a.rope && (geo.G + 2u) * (a.head_dim / 8u) > kAttnThreads) {
        // More heads than one CTA's threads hold: the rope launch first, then
        // the attention over its output, as without the fused form.
        if (cudaError_t e = rope_run(*a.rope, stream, pdl); e != cudaSuccess) return e;
        AttentionArgs b = a;
        b.query = a.rope->query;
        b.rope = nullptr;
        return attention_run(b, stream, pdl);
    }
    const size_t base_smem = attention_smem(a.head_dim, kMaxQueries);
    if (base_smem > 200u * 1024u) return cudaErrorInvalidValue;
    // A one-token decode step may fold over a cluster, with room in rank 0
    // for every chunk's partial; so may batched sequences whose CTAs all fit
    // one wave, on a layer whose window's chunks always fit the cluster (a
    // step past that would fold globally inside a cluster launch, slower).
    // Larger batches keep the global fold: the fold room would halve the
    // CTAs an SM holds across their many row tiles.
    // Decode shapes on a sliding-window layer take only as many chunk slots
    // as the window's keys can span (a 512-key window: 9), so a cluster holds
    // no CTA that can never have a chunk, and a launch no CTA that only leaves.
    const uint32_t all_slots = a.max_chunks < kChunkSlots ? a.max_chunks : kChunkSlots;
    const uint32_t window_chunks = a.window / kChunk + 1u + (a.window % kChunk ? 1u : 0u);
    const uint32_t slots = window_chunks < all_slots ? window_chunks : all_slots;
    const int sms = sm_count();
    const bool decode_shape =
        a.tokens == 1u || (a.rows_are_sequences && sms > 0 && a.window / kChunk + 1u <= slots &&
                           static_cast<uint64_t>(a.kv_heads) * slots * a.tokens <= static_cast<uint64_t>(sms));
    // Batched sequences keep the window's slots in the global fold too (a
    // row a tile: its live chunks never span more); tiles of several rows
    // take every slot.
    const uint32_t launch_slots = decode_shape || a.rows_are_sequences ? slots : all_slots;
    const size_t cluster_smem = base_smem + cluster_fold_floats(a.head_dim, geo.G) * 4u;
    return a.head_dim == 64 ? launch_attention<64>(a, stream, pdl, base_smem, cluster_smem, decode_shape, launch_slots)
           : a.head_dim == 128 ? launch_attention<128>(a, stream, pdl, base_smem, cluster_smem, decode_shape, launch_slots)
                               : launch_attention<256>(a, stream, pdl, base_smem, cluster_smem, decode_shape, launch_slots);
}

}  // namespace cb
