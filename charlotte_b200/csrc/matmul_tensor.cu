// The tensor-core form of the matrix products (CB_MATMUL_TENSOR): Y = X·Wᵀ
// for steps of many tokens on the 5th-generation tensor cores, at the
// BASELINE tolerance tier (max |y − y_exact| ≤ 1e-3·max |y|), not bit-exact:
// X and the decoded weights are rounded to f16 (round to nearest even) and
// the products accumulate in f32 in tensor memory, in the tensor core's own
// order. Each weight is decoded exactly (formats.cuh) before that rounding.
// Inputs beyond ±65,504 do not fit f16; the exact forms serve those.
//
// B200 mapping, two launches:
//  1. x is rounded to f16 once, into the caller's scratch ([tokens][K]);
//  2. one CTA a 128-token × 128-slot tile:
//     - a TMA warp loads each 128 × 64 block of x16 with a tiled bulk tensor
//       copy (128-byte swizzle, this CTA only) straight into the K-major
//       layout the MMA reads;
//     - eight producer warps decode the tile's weight blocks (four blocks of
//       codes in flight in registers a thread) to f16 and store them in the
//       same swizzled layout;
//     - one warp issues tcgen05.mma (M = 128, N = 128, K = 16, four a block)
//       into a 128-column f32 accumulator in tensor memory; tcgen05.commit
//       hands each of the 6 ring stages back;
//     - after the last block the producer warps read the accumulator
//       (tcgen05.ld) and apply the epilogue: write, QKV, gated (the tile's
//       first 64 slots are gate rows, the last 64 the same outputs' up rows)
//       or gated by input.
// Every wait is bounded; a wait that runs out sets the fault word, the
// pipeline drains, and the accumulator is still freed.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <utility>

#include "formats.cuh"
#include "matmul.h"
#include "numerics.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace cb {

namespace {

constexpr uint32_t kBM = 128, kBN = 128, kBK = 64, kStages = 6;
constexpr uint32_t kProducerWarps = 8, kProducers = kProducerWarps * 32;
constexpr uint32_t kMmaWarp = kProducerWarps, kTmaWarp = kProducerWarps + 1;
constexpr uint32_t kThreadsT = kProducers + 64;                 // + the MMA warp and the TMA warp
constexpr uint32_t kTileA = kBM * kBK * 2, kTileB = kBN * kBK * 2;   // 16 KB each
constexpr uint32_t kStageBytes = kTileA + kTileB;
constexpr uint32_t kTmemColumns = 128;
constexpr size_t kTensorSmem = 1024 + kStages * kStageBytes + 256;

// Byte offset of 16-byte chunk c of row r in a K-major 128-byte-swizzled tile.
__device__ __forceinline__ uint32_t sw128(uint32_t r, uint32_t c) { return r * 128u + ((c ^ (r & 7u)) << 4); }

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// Weights [K0, K0+16) of a group, exactly decoded, as eight packed f16 pairs.
template <typename F, int K0, int... ks>
__device__ __forceinline__ void decode16(const F& f, const typename F::Consts& c, uint32_t (&h)[8],
                                         std::integer_sequence<int, ks...>) {
    float w[16];
    ((w[ks] = F::template weight<K0 + ks>(f, c)), ...);
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = pack_half2(w[2 * i], w[2 * i + 1]);
}

// x rounded to f16 (round to nearest even), [tokens][K].
__global__ void to_f16_kernel(const float* x, uint32_t x_stride, uint32_t K, uint32_t tokens, __half2* x16) {
    grid_dependency_wait();
    const uint32_t quads = K / 4u;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < tokens * quads; i += gridDim.x * blockDim.x) {
        const uint32_t t = i / quads, q = i % quads;
        const float4 v = __ldcg(reinterpret_cast<const float4*>(x + static_cast<size_t>(t) * x_stride) + q);
        x16[2u * i] = __floats2half2_rn(v.x, v.y);
        x16[2u * i + 1u] = __floats2half2_rn(v.z, v.w);
    }
    grid_dependents_launch();
}

// Tiled TMA load of box {64, 128} at (k0, row0) of the x16 map into `dst`,
// completing on `bar`, into this CTA's shared memory only.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int32_t k0, int32_t row0,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(k0), "r"(row0), "r"(smem_addr(bar))
        : "memory");
}

template <typename F>
__global__ void __launch_bounds__(kThreadsT, 1) tensor_kernel(const MatmulArgs a, const __grid_constant__ CUtensorMap x16map) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023u) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(base + kStages * kStageBytes);
    uint64_t* empty = full + kStages;
    uint64_t* done = empty + kStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t G = a.columns / 32u;
    const uint32_t kblocks = (G + 1u) / 2u;
    const bool gated = a.epilogue == kGated;
    const uint32_t m0 = blockIdx.x * kBM;
    const uint32_t n0 = blockIdx.y * (gated ? kBN / 2 : kBN);   // first slot (gated: first output)

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < kStages; ++s) {
            mbar_init(&full[s], kProducers + 1u);   // the producers, and the TMA warp's expect-tx
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, kTmemColumns);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    grid_dependency_wait();

    if (warp < kProducerWarps) {
        // ---- producers: row r of B, half h of each K block ---------------------
        const uint32_t tid = threadIdx.x;
        const uint32_t r = tid % 128u, h = tid / 128u;
        // B: slot r's weight row (members picked by value, see matmul_tiled.cu).
        const uint8_t* sp[F::kStreams];
        bool live = false;
        {
            int q = -1;
            uint32_t row = 0;
            if (gated) {
                const uint32_t o = n0 + (r < kBN / 2 ? r : r - kBN / 2);
                if (o < a.member[0].rows) {
                    q = r < kBN / 2 ? 0 : 1;
                    row = (q == 0 ? a.member[0].first_row : a.member[1].first_row) + o;
                }
            } else {
                uint32_t n = n0 + r;
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
        // Eight blocks' codes in flight in registers: block kb+8 is read from
        // global memory while block kb is decoded and stored.
        auto fetch = [&](uint32_t kb, F& f) {
            const uint32_t g = 2u * kb + h;   // this thread's 32-wide group of the block
            if (live && g < G) f.load(sp, g);
            else f.zero();
        };
        // Stores block kb (stage kb mod kStages): the slot's group decoded
        // exactly and rounded to f16, as four 16-byte swizzled chunks.
        auto put = [&](uint32_t kb, const F& f) -> bool {
            const uint32_t s = kb % kStages;
            if (kb >= kStages && !mbar_wait(&empty[s], ((kb / kStages) - 1u) & 1u, a.fault)) return false;
            uint8_t* tileB = base + s * kStageBytes + kTileA;
            const typename F::Consts c = f.consts();
            uint32_t lo[8], hi[8];
            decode16<F, 0>(f, c, lo, std::make_integer_sequence<int, 16>{});
            decode16<F, 16>(f, c, hi, std::make_integer_sequence<int, 16>{});
            *reinterpret_cast<uint4*>(tileB + sw128(r, 4u * h + 0)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            *reinterpret_cast<uint4*>(tileB + sw128(r, 4u * h + 1)) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
            *reinterpret_cast<uint4*>(tileB + sw128(r, 4u * h + 2)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
            *reinterpret_cast<uint4*>(tileB + sw128(r, 4u * h + 3)) = make_uint4(hi[4], hi[5], hi[6], hi[7]);
            fence_proxy_async();   // generic-proxy stores, then the tensor core's reads
            mbar_arrive(&full[s]);
            return true;
        };
        F f[8];
#pragma unroll
        for (uint32_t j = 0; j < 8u; ++j) fetch(j, f[j]);
        bool running = true;
        for (uint32_t kb = 0; kb < kblocks && running; kb += 8u) {
#pragma unroll
            for (uint32_t j = 0; j < 8u; ++j) {
                if (kb + j >= kblocks || !put(kb + j, f[j])) { running = false; break; }
                fetch(kb + j + 8u, f[j]);
            }
        }
    } else if (warp == kTmaWarp) {
        // ---- the TMA warp: x16 blocks ------------------------------------------
        if (lane == 0) {
            for (uint32_t kb = 0; kb < kblocks; ++kb) {
                const uint32_t s = kb % kStages;
                if (kb >= kStages && !mbar_wait(&empty[s], ((kb / kStages) - 1u) & 1u, a.fault)) break;
                mbar_arrive_expect_tx(&full[s], kTileA);
                tma_load_2d(base + s * kStageBytes, &x16map, static_cast<int32_t>(kb * kBK), static_cast<int32_t>(m0),
                            &full[s]);
            }
        }
        __syncwarp();
    } else {
        // ---- the MMA warp ---------------------------------------------------------
        constexpr uint32_t idesc = umma_idesc_f16(kBM, kBN);
        for (uint32_t kb = 0; kb < kblocks; ++kb) {
            const uint32_t s = kb % kStages;
            if (!mbar_wait(&full[s], (kb / kStages) & 1u, a.fault)) break;
            tc_fence_after();
            if (lane == 0) {
                const uint32_t a_addr = smem_addr(base + s * kStageBytes);
                const uint64_t da = umma_desc_sw128(a_addr), db = umma_desc_sw128(a_addr + kTileA);
#pragma unroll
                for (uint32_t kk = 0; kk < kBK / 16u; ++kk)   // 32 bytes of K an MMA
                    umma_f16(tmem, da + 2u * kk, db + 2u * kk, idesc, (kb | kk) != 0u ? 1u : 0u);
                umma_commit(&empty[s]);
            }
            __syncwarp();
        }
        if (lane == 0) umma_commit(done);   // when every MMA issued has completed
        __syncwarp();
    }
    grid_dependents_launch();

    // ---- epilogue: producer warp w reads TMEM lanes 32·(w mod 4), columns
    //      [32·(w/4), +32) and [64 + 32·(w/4), +32), into a 128 × 128 tile in
    //      the drained ring; then each warp writes whole output rows, its
    //      lanes over consecutive columns (coalesced) ------------------------
    if (warp < kProducerWarps) {
        const bool ok = mbar_wait(done, 0u, a.fault);
        constexpr uint32_t kCs = kBN + 1u;   // floats a staged row: conflict-free column writes
        float* cs = reinterpret_cast<float*>(base);
        if (ok) {
            tc_fence_after();
            const uint32_t quarter = warp & 3u, half = warp >> 2;
            const uint32_t row = 32u * quarter + lane;
            float lo[32], hi[32];
            const uint32_t lane_addr = tmem + ((32u * quarter) << 16);
            tmem_ld32(lane_addr + 32u * half, lo);
            tmem_ld32(lane_addr + 64u + 32u * half, hi);
            fence_proxy_async();   // the ring was last written by the copy engine and read by the MMA
#pragma unroll
            for (uint32_t c = 0; c < 32; ++c) {
                cs[row * kCs + 32u * half + c] = lo[c];
                cs[row * kCs + 64u + 32u * half + c] = hi[c];
            }
        }
        asm volatile("bar.sync 1, %0;" ::"n"(kProducers) : "memory");
        if (ok) {
            if (gated) {
                for (uint32_t r = warp; r < kBM && m0 + r < a.tokens; r += kProducerWarps) {
                    const size_t rowbase = static_cast<size_t>(m0 + r) * a.out_stride[0] + a.member[0].out_offset;
#pragma unroll
                    for (uint32_t j = 0; j < 2; ++j) {
                        const uint32_t c = lane + 32u * j, o = n0 + c;
                        if (o < a.member[0].rows)
                            a.out[0][rowbase + o] = activate(a.activation, cs[r * kCs + c]) * cs[r * kCs + 64u + c];
                    }
                }
            } else {
                // Column lane + 32j of the tile: its member and output column.
                int qj[4];
                uint32_t oj[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    uint32_t n = n0 + lane + 32u * j;
                    int q = -1;
#pragma unroll
                    for (int m = 0; m < 3; ++m) {
                        if (q < 0 && m < static_cast<int>(a.members)) {
                            if (n < a.member[m].rows) q = m;
                            else n -= a.member[m].rows;
                        }
                    }
                    qj[j] = q;
                    oj[j] = (q == 1 ? a.member[1].out_offset : (q == 2 ? a.member[2].out_offset : a.member[0].out_offset)) + n;
                }
                for (uint32_t r = warp; r < kBM && m0 + r < a.tokens; r += kProducerWarps) {
                    const uint32_t t = m0 + r;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int q = qj[j];
                        if (q < 0) continue;
                        const float v = cs[r * kCs + lane + 32u * j];
                        const uint32_t o = oj[j];
                        if (a.epilogue == kQKV) {
                            float* out = q == 1 ? a.out[1] : (q == 2 ? a.out[2] : a.out[0]);
                            const uint32_t st = q == 1 ? a.out_stride[1] : (q == 2 ? a.out_stride[2] : a.out_stride[0]);
                            out[static_cast<size_t>(t) * st + o] = v;
                        } else if (a.epilogue == kWrite) {
                            a.out[0][static_cast<size_t>(t) * a.out_stride[0] + o] = v;
                        } else {   // kGatedByInput
                            const float u = a.gate_input[static_cast<size_t>(a.token + t) * a.gate_input_stride +
                                                         a.gate_input_column + o];
                            a.out[0][static_cast<size_t>(t) * a.out_stride[0] + o] = activate(a.activation, v) * u;
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemColumns);
    }
}

template <typename F>
cudaError_t launch_tensor(const MatmulArgs& a, const CUtensorMap& map, cudaStream_t stream, bool pdl) {
    auto kernel = tensor_kernel<F>;
    static bool configured = false;
    if (!configured) {
        cudaError_t e =
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kTensorSmem));
        if (e != cudaSuccess) return e;
        configured = true;
    }
    const bool gated = a.epilogue == kGated;
    const uint32_t slots = gated ? a.member[0].rows : a.total_rows;
    const uint32_t per_tile = gated ? kBN / 2 : kBN;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((a.tokens + kBM - 1) / kBM, (slots + per_tile - 1) / per_tile);
    cfg.blockDim = dim3(kThreadsT);
    cfg.dynamicSmemBytes = kTensorSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, a, map);
}

// x rounded to f16 into the scratch.
cudaError_t launch_to_f16(const MatmulArgs& a, cudaStream_t stream, bool pdl) {
    const uint32_t quads = a.tokens * (a.columns / 4u);
    uint32_t blocks = (quads + 255u) / 256u;
    if (blocks > 4096u) blocks = 4096u;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks);
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, to_f16_kernel, a.x, a.x_stride, a.columns, a.tokens,
                              static_cast<__half2*>(a.scratch));
}

// The map of an f16 [rows][K] matrix: boxes of 64 × box_rows with the
// 128-byte swizzle; rows past `rows` and columns past K read as zero. The
// driver's encoder is looked up through the runtime once (the library does
// not link the driver library, so it still loads where there is no GPU
// driver).
cudaError_t encode_f16_map(CUtensorMap* map, const void* base, uint32_t K, uint32_t rows, uint32_t box_rows) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    if (!encode) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !fn)
            return cudaErrorNotSupported;
        encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    const cuuint64_t dims[2] = {K, rows};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2u};
    const cuuint32_t box[2] = {kBK, box_rows};
    const cuuint32_t elem[2] = {1, 1};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                              elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}


// ---- the dense form ----------------------------------------------------------
//
// The product's weights are decoded once (exactly, then rounded to f16) into
// a dense [slots][K] matrix — at load time by a runtime that keeps it, or
// once per call — so the GEMM streams both operands by TMA and the tensor
// core is fed without producer warps. Slot order: the members' rows one
// after another; a gated product interleaves 64-slot units, 64 outputs'
// gate rows then the same outputs' up rows, so any 128-slot-aligned tile
// holds whole (gate, up) pairs. Padding slots are zero rows.

// Slot s's member (-1: a zero row) and weight row.
struct SlotRow {
    int q;
    uint32_t row;
};
__device__ __forceinline__ SlotRow slot_row(const MatmulArgs& a, uint32_t s) {
    if (a.epilogue == kGated) {
        const uint32_t unit = s / 64u, o = (unit / 2u) * 64u + s % 64u;
        if (o >= a.member[0].rows) return {-1, 0u};
        return (unit & 1u) ? SlotRow{1, a.member[1].first_row + o} : SlotRow{0, a.member[0].first_row + o};
    }
    uint32_t n = s;
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        if (i < static_cast<int>(a.members)) {
            const uint32_t rows = i == 0 ? a.member[0].rows : (i == 1 ? a.member[1].rows : a.member[2].rows);
            if (n < rows) {
                const uint32_t first = i == 0 ? a.member[0].first_row : (i == 1 ? a.member[1].first_row : a.member[2].first_row);
                return {i, first + n};
            }
            n -= rows;
        }
    }
    return {-1, 0u};
}

__host__ __device__ __forceinline__ uint32_t dense_slot_count(const MatmulArgs& a) {
    return a.epilogue == kGated ? 128u * ((a.member[0].rows + 63u) / 64u) : a.total_rows;
}

// A warp a slot row: each lane decodes 32-weight groups and stores them as
// 64 contiguous bytes of f16.
template <typename F>
__global__ void __launch_bounds__(256) densify_kernel(const MatmulArgs a, uint32_t slots, uint4* dense) {
    const uint32_t G = a.columns / 32u, lane = threadIdx.x & 31u;
    const uint32_t warps = blockDim.x / 32u;
    for (uint32_t s = blockIdx.x * warps + threadIdx.x / 32u; s < slots; s += gridDim.x * warps) {
        uint4* dst = dense + static_cast<size_t>(s) * (a.columns / 8u);
        const SlotRow sr = slot_row(a, s);
        if (sr.q < 0) {
            for (uint32_t g = lane; g < G; g += 32u)
#pragma unroll
                for (int i = 0; i < 4; ++i) dst[4u * g + i] = make_uint4(0u, 0u, 0u, 0u);
            continue;
        }
        const uint8_t* piece = sr.q == 1 ? a.member[1].piece : (sr.q == 2 ? a.member[2].piece : a.member[0].piece);
        const uint32_t blocks = sr.q == 1 ? a.member[1].blocks : (sr.q == 2 ? a.member[2].blocks : a.member[0].blocks);
        const uint8_t* sp[F::kStreams];
#pragma unroll
        for (int q = 0; q < F::kStreams; ++q)
            sp[q] = piece + RowStreams<F>::base(q, blocks) + static_cast<uint64_t>(sr.row) * RowStreams<F>::row_bytes(q, G);
        for (uint32_t g = lane; g < G; g += 32u) {
            F f;
            f.load(sp, g);
            const typename F::Consts c = f.consts();
            uint32_t lo[8], hi[8];
            decode16<F, 0>(f, c, lo, std::make_integer_sequence<int, 16>{});
            decode16<F, 16>(f, c, hi, std::make_integer_sequence<int, 16>{});
            dst[4u * g + 0] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            dst[4u * g + 1] = make_uint4(lo[4], lo[5], lo[6], lo[7]);
            dst[4u * g + 2] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
            dst[4u * g + 3] = make_uint4(hi[4], hi[5], hi[6], hi[7]);
        }
    }
}

// Output of non-gated slot n for token t: its member's output and column.
__device__ __forceinline__ void put_slot(const MatmulArgs& a, uint32_t t, uint32_t n, float v) {
    int q = -1;
#pragma unroll
    for (int m = 0; m < 3; ++m) {
        if (q < 0 && m < static_cast<int>(a.members)) {
            const uint32_t rows = m == 0 ? a.member[0].rows : (m == 1 ? a.member[1].rows : a.member[2].rows);
            if (n < rows) q = m;
            else n -= rows;
        }
    }
    if (q < 0) return;
    const uint32_t o = (q == 1 ? a.member[1].out_offset : (q == 2 ? a.member[2].out_offset : a.member[0].out_offset)) + n;
    if (a.epilogue == kQKV) {
        float* out = q == 1 ? a.out[1] : (q == 2 ? a.out[2] : a.out[0]);
        const uint32_t st = q == 1 ? a.out_stride[1] : (q == 2 ? a.out_stride[2] : a.out_stride[0]);
        out[static_cast<size_t>(t) * st + o] = v;
    } else if (a.epilogue == kWrite) {
        a.out[0][static_cast<size_t>(t) * a.out_stride[0] + o] = v;
    } else {   // kGatedByInput
        const float u =
            a.gate_input[static_cast<size_t>(a.token + t) * a.gate_input_stride + a.gate_input_column + o];
        a.out[0][static_cast<size_t>(t) * a.out_stride[0] + o] = activate(a.activation, v) * u;
    }
}

__device__ __forceinline__ void put_gated(const MatmulArgs& a, uint32_t t, uint32_t o, float g, float u) {
    const size_t at = static_cast<size_t>(t) * a.out_stride[0] + a.member[0].out_offset + o;
    const float v = activate(a.activation, g) * u;
    a.out[0][at] = v;
    if (a.out16) static_cast<__half*>(a.out16)[at] = __float2half_rn(v);
}

template <uint32_t BN>
struct Dense {
    static constexpr uint32_t kA = kBM * kBK * 2;                 // 16 KB of x16
    static constexpr uint32_t kB = BN * kBK * 2;                  // 16 KB of weights (BN = 128)
    static constexpr uint32_t kStage = kA + kB;
    static constexpr uint32_t kStages = (192u * 1024u) / kStage;
    static constexpr uint32_t kCs = BN + 1;                       // floats a staged row
    static constexpr uint32_t kWarps = 8;
    static constexpr size_t kSmem = 1024 + kStages * kStage + 256;
    static_assert(kBM * kCs * 4 <= kStages * kStage, "the staged tile fits the drained ring");
};

// One CTA a 128-token × BN-slot tile over K blocks [kb0, kb1) of split z,
// for products of too few tiles for the persistent form. Warp 0's lane 0
// loads the operands by TMA (the first stages' weights before the wait on
// the previous kernel, which they do not depend on), warp 1's lane 0 issues
// the MMAs (M = 128, N = BN, K = 16; four a block) into a BN-column f32
// accumulator in tensor memory, and the eight warps read it back (warp w:
// lanes 32·(w mod 4), half w/4 of the columns) through shared memory into
// coalesced row writes: the epilogue, or split z's raw partial tile.
template <uint32_t BN>
__global__ void __launch_bounds__(256, 1)
    dense_kernel(const MatmulArgs a, const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                 uint32_t splits, float* partials) {
    using S = Dense<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023u) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(base + S::kStages * S::kStage);
    uint64_t* empty = full + S::kStages;
    uint64_t* done = empty + S::kStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t all_blocks = (a.columns + kBK - 1u) / kBK;
    const uint32_t kb0 = all_blocks * blockIdx.z / splits, kb1 = all_blocks * (blockIdx.z + 1u) / splits;
    const uint32_t kblocks = kb1 - kb0;
    const uint32_t m0 = blockIdx.x * kBM, n0 = blockIdx.y * BN;
    const uint32_t slots = dense_slot_count(a);

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < S::kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, BN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            auto load_x = [&](uint32_t s, uint32_t kb) {
                tma_load_2d(base + s * S::kStage, &xmap, static_cast<int32_t>((kb0 + kb) * kBK), static_cast<int32_t>(m0),
                            &full[s]);
            };
            const uint32_t pre = kblocks < S::kStages ? kblocks : S::kStages;
            for (uint32_t i = 0; i < pre; ++i) {
                mbar_arrive_expect_tx(&full[i], S::kStage);
                tma_load_2d(base + i * S::kStage + S::kA, &wmap, static_cast<int32_t>((kb0 + i) * kBK),
                            static_cast<int32_t>(n0), &full[i]);
            }
            grid_dependency_wait();   // x16 is the previous kernel's output
            for (uint32_t i = 0; i < pre; ++i) load_x(i, i);
            uint32_t issued = pre;
            for (uint32_t kb = pre; kb < kblocks; ++kb) {
                const uint32_t s = kb % S::kStages;
                if (!mbar_wait(&empty[s], ((kb / S::kStages) - 1u) & 1u, a.fault)) break;
                mbar_arrive_expect_tx(&full[s], S::kStage);
                load_x(s, kb);
                tma_load_2d(base + s * S::kStage + S::kA, &wmap, static_cast<int32_t>((kb0 + kb) * kBK),
                            static_cast<int32_t>(n0), &full[s]);
                issued = kb + 1u;
            }
            // Every copy issued has landed before this CTA's shared memory is
            // reused or released (immediate unless a wait above ran out).
            for (uint32_t kb = issued > S::kStages ? issued - S::kStages : 0u; kb < issued; ++kb)
                mbar_wait(&full[kb % S::kStages], (kb / S::kStages) & 1u, nullptr);
        }
        __syncwarp();
    } else {
        grid_dependency_wait();
        if (warp == 1) {
            constexpr uint32_t idesc = umma_idesc_f16(kBM, BN);
            for (uint32_t kb = 0; kb < kblocks; ++kb) {
                const uint32_t s = kb % S::kStages;
                if (!mbar_wait(&full[s], (kb / S::kStages) & 1u, a.fault)) break;
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t stage = smem_addr(base + s * S::kStage);
                    const uint64_t da = umma_desc_sw128(stage), db = umma_desc_sw128(stage + S::kA);
#pragma unroll
                    for (uint32_t kk = 0; kk < kBK / 16u; ++kk)
                        umma_f16(tmem, da + 2u * kk, db + 2u * kk, idesc, (kb | kk) != 0u ? 1u : 0u);
                    umma_commit(&empty[s]);
                }
                __syncwarp();
            }
            if (lane == 0) umma_commit(done);
            __syncwarp();
        }
    }
    grid_dependents_launch();

    const bool ok = mbar_wait(done, 0u, a.fault);
    float* cs = reinterpret_cast<float*>(base);
    const uint32_t quarter = warp & 3u, half = warp >> 2;
    if (ok) {
        tc_fence_after();
        fence_proxy_async();   // the ring was last written by the copy engine
        const uint32_t row = 32u * quarter + lane;
        const uint32_t taddr = tmem + ((32u * quarter) << 16);
#pragma unroll 1
        for (uint32_t c0 = half * (BN / 2u); c0 < (half + 1u) * (BN / 2u); c0 += 32u) {
            float v[32];
            tmem_ld32(taddr + c0, v);
#pragma unroll
            for (uint32_t i = 0; i < 32u; ++i) cs[row * S::kCs + c0 + i] = v[i];
        }
    }
    __syncthreads();
    if (ok && m0 < a.tokens) {
        if (splits > 1u) {
            // split z's raw sums: partials[(z·tokens + t)·slots + n]
            for (uint32_t r = warp; r < kBM && m0 + r < a.tokens; r += S::kWarps) {
                float* dst = partials + (static_cast<size_t>(blockIdx.z) * a.tokens + m0 + r) * slots;
#pragma unroll
                for (uint32_t j = 0; j < BN / 32u; ++j) {
                    const uint32_t n = n0 + lane + 32u * j;
                    if (n < slots) dst[n] = cs[r * S::kCs + lane + 32u * j];
                }
            }
        } else if (a.epilogue == kGated) {
            // the tile's outputs: BN/2, unit pairs (gate 64, up 64)
            for (uint32_t r = warp; r < kBM && m0 + r < a.tokens; r += S::kWarps) {
#pragma unroll
                for (uint32_t j = 0; j < BN / 64u; ++j) {
                    const uint32_t c = lane + 32u * j, gc = (c / 64u) * 128u + c % 64u;
                    const uint32_t o = n0 / 2u + c;
                    if (o < a.member[0].rows)
                        put_gated(a, m0 + r, o, cs[r * S::kCs + gc], cs[r * S::kCs + gc + 64u]);
                }
            }
        } else {
            for (uint32_t r = warp; r < kBM && m0 + r < a.tokens; r += S::kWarps) {
#pragma unroll
                for (uint32_t j = 0; j < BN / 32u; ++j) {
                    const uint32_t n = n0 + lane + 32u * j;
                    if (n < slots) put_slot(a, m0 + r, n, cs[r * S::kCs + lane + 32u * j]);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, BN);
    }
}

// ---- the persistent dense form: products of at least a wave of tiles ------

// Waits like mbar_wait, and gives up early once another role of the CTA has
// given up (`abort`, in shared memory): a wait that runs out sets the fault
// word and `abort`, so the other roles leave within a few hundred polls.
__device__ __forceinline__ bool role_wait(uint64_t* bar, uint32_t parity, unsigned int* fault,
                                          volatile uint32_t* abort) {
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 255u && *abort) return false;
    }
    if (fault) atomicOr(fault, kFaultTimeout);
    *abort = 1u;
    return false;
}

// A 32 × 32 block of outputs — tokens t0 + r (r = 0..31) × slots
// [n, n + 32) — from registers (lane r holding its token's 32 values) to
// the outputs through the warp's staging buffer `stg` (32 rows of 33
// floats: conflict-free both ways), so each store instruction writes 32
// consecutive floats of one token's row. The Write and QKV epilogues write
// straight when one member holds the 32 slots; otherwise each slot takes
// put_slot.
__device__ __forceinline__ void store_block(const MatmulArgs& a, uint32_t t0, uint32_t n, const float (&v)[32],
                                            uint32_t slots, float* stg, uint32_t lane) {
#pragma unroll
    for (uint32_t i = 0; i < 32u; ++i) stg[lane * 33u + i] = v[i];
    __syncwarp();
    int q = -1;
    uint32_t local = n, rows = 0;
#pragma unroll
    for (int m = 0; m < 3; ++m) {
        if (q < 0 && m < static_cast<int>(a.members)) {
            const uint32_t r = m == 0 ? a.member[0].rows : (m == 1 ? a.member[1].rows : a.member[2].rows);
            if (local < r) {
                q = m;
                rows = r;
            } else {
                local -= r;
            }
        }
    }
    const uint32_t live = a.tokens > t0 ? (a.tokens - t0 < 32u ? a.tokens - t0 : 32u) : 0u;
    if (q >= 0 && local + 32u <= rows && a.epilogue != kGatedByInput) {
        const bool qkv = a.epilogue == kQKV;
        float* out = qkv ? (q == 1 ? a.out[1] : (q == 2 ? a.out[2] : a.out[0])) : a.out[0];
        const uint32_t st = qkv ? (q == 1 ? a.out_stride[1] : (q == 2 ? a.out_stride[2] : a.out_stride[0])) : a.out_stride[0];
        const uint32_t off = q == 1 ? a.member[1].out_offset : (q == 2 ? a.member[2].out_offset : a.member[0].out_offset);
        float* dst = out + static_cast<size_t>(t0) * st + off + local + lane;
        for (uint32_t r = 0; r < live; ++r) dst[static_cast<size_t>(r) * st] = stg[r * 33u + lane];
    } else if (n + lane < slots) {
        for (uint32_t r = 0; r < live; ++r) put_slot(a, t0 + r, n + lane, stg[r * 33u + lane]);
    }
    __syncwarp();   // the staging buffer is read before the next block
}

struct Persist {
    static constexpr uint32_t kBN = 256;
    static constexpr uint32_t kA = kBM * kBK * 2;      // 16 KB of x16
    static constexpr uint32_t kB = kBN * kBK * 2;      // 32 KB of weights
    static constexpr uint32_t kStage = kA + kB;
    static constexpr uint32_t kStages = 4;
    static constexpr uint32_t kEpilogueWarps = 8;
    static constexpr uint32_t kThreads = 32u * (2u + kEpilogueWarps);
    static constexpr uint32_t kStaging = 32u * 33u * 4u;   // bytes an epilogue warp stages a block in
    static constexpr size_t kSmem = 1024 + kStages * kStage + 256 + kEpilogueWarps * kStaging;
};

// A CTA an SM, looping over the product's 128-token × 256-slot tiles (tile
// blockIdx.x, then every gridDim.x-th; token tiles fastest, so the CTAs at
// work together share weight tiles in L2). Warp 0's lane 0 streams both
// operands by TMA through a 4-stage ring across tiles; warp 1's lane 0
// issues the MMAs into one of two 256-column accumulators in tensor memory,
// alternating by tile; warps 2-9 drain the other accumulator at the same
// time (warp w: lanes 32·(w mod 4), half (w − 2)/4 of the columns), from
// registers straight to the outputs, then hand it back.
__global__ void __launch_bounds__(Persist::kThreads, 1)
    dense_persistent_kernel(const MatmulArgs a, const __grid_constant__ CUtensorMap xmap,
                            const __grid_constant__ CUtensorMap wmap) {
    using P = Persist;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023u) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(base + P::kStages * P::kStage);
    uint64_t* empty = full + P::kStages;
    uint64_t* acc_full = empty + P::kStages;   // [2]: an accumulator is complete
    uint64_t* acc_empty = acc_full + 2;        // [2]: an accumulator is drained
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    volatile uint32_t* abort = tmem_slot + 1;
    float* staging = reinterpret_cast<float*>(base + P::kStages * P::kStage + 256);

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t slots = dense_slot_count(a);
    const uint32_t kblocks = (a.columns + kBK - 1u) / kBK;
    const uint32_t m_tiles = (a.tokens + kBM - 1u) / kBM, n_tiles = (slots + P::kBN - 1u) / P::kBN;
    const uint32_t tiles = m_tiles * n_tiles;
    const uint32_t mine = tiles > blockIdx.x ? (tiles - blockIdx.x + gridDim.x - 1u) / gridDim.x : 0u;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < P::kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (uint32_t b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], P::kEpilogueWarps);
        }
        *abort = 0u;
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, 2u * P::kBN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            const uint32_t total = mine * kblocks;
            auto tile_of = [&](uint32_t g) { return blockIdx.x + (g / kblocks) * gridDim.x; };
            auto load_w = [&](uint32_t g, uint32_t s) {
                tma_load_2d(base + s * P::kStage + P::kA, &wmap, static_cast<int32_t>((g % kblocks) * kBK),
                            static_cast<int32_t>((tile_of(g) / m_tiles) * P::kBN), &full[s]);
            };
            auto load_x = [&](uint32_t g, uint32_t s) {
                tma_load_2d(base + s * P::kStage, &xmap, static_cast<int32_t>((g % kblocks) * kBK),
                            static_cast<int32_t>((tile_of(g) % m_tiles) * kBM), &full[s]);
            };
            // The first stages' weights before the wait on the previous
            // kernel (x16 is its output; the weights do not depend on it).
            const uint32_t pre = total < P::kStages ? total : P::kStages;
            for (uint32_t g = 0; g < pre; ++g) {
                mbar_arrive_expect_tx(&full[g], P::kStage);
                load_w(g, g);
            }
            grid_dependency_wait();
            for (uint32_t g = 0; g < pre; ++g) load_x(g, g);
            uint32_t issued = pre;
            for (uint32_t g = pre; g < total; ++g) {
                const uint32_t s = g % P::kStages;
                if (!role_wait(&empty[s], ((g / P::kStages) - 1u) & 1u, a.fault, abort)) break;
                mbar_arrive_expect_tx(&full[s], P::kStage);
                load_x(g, s);
                load_w(g, s);
                issued = g + 1u;
            }
            // Every copy issued has landed before the CTA leaves.
            for (uint32_t g = issued > P::kStages ? issued - P::kStages : 0u; g < issued; ++g)
                mbar_wait(&full[g % P::kStages], (g / P::kStages) & 1u, nullptr);
        }
        __syncwarp();
    } else if (warp == 1) {
        constexpr uint32_t idesc = umma_idesc_f16(kBM, P::kBN);
        uint32_t g = 0;
        bool ok = true;
        for (uint32_t i = 0; i < mine && ok; ++i) {
            const uint32_t b = i & 1u;
            if (i >= 2u) {
                bool got = lane == 0 ? role_wait(&acc_empty[b], ((i >> 1) - 1u) & 1u, a.fault, abort) : false;
                if (!__shfl_sync(0xFFFFFFFFu, got, 0)) break;
                tc_fence_after();
            }
            for (uint32_t kb = 0; kb < kblocks; ++kb, ++g) {
                const uint32_t s = g % P::kStages;
                bool got = lane == 0 ? role_wait(&full[s], (g / P::kStages) & 1u, a.fault, abort) : false;
                if (!__shfl_sync(0xFFFFFFFFu, got, 0)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t stage = smem_addr(base + s * P::kStage);
                    const uint64_t da = umma_desc_sw128(stage), db = umma_desc_sw128(stage + P::kA);
#pragma unroll
                    for (uint32_t kk = 0; kk < kBK / 16u; ++kk)
                        umma_f16(tmem + b * P::kBN, da + 2u * kk, db + 2u * kk, idesc, (kb | kk) != 0u ? 1u : 0u);
                    umma_commit(&empty[s]);
                }
                __syncwarp();
            }
            // Complete even after a failed wait: the epilogue's wait ends.
            if (lane == 0) umma_commit(&acc_full[b]);
            __syncwarp();
        }
    } else {
        grid_dependency_wait();
        const uint32_t quarter = warp & 3u, part = (warp - 2u) / 4u;
        for (uint32_t i = 0; i < mine; ++i) {
            const uint32_t b = i & 1u;
            const uint32_t tile = blockIdx.x + i * gridDim.x;
            const uint32_t m0 = (tile % m_tiles) * kBM, n0 = (tile / m_tiles) * P::kBN;
            bool got = lane == 0 ? role_wait(&acc_full[b], (i >> 1) & 1u, a.fault, abort) : false;
            if (!__shfl_sync(0xFFFFFFFFu, got, 0)) break;
            tc_fence_after();
            const uint32_t t0 = m0 + 32u * quarter;   // the warp's 32 tokens, lane = token
            const uint32_t taddr = tmem + ((32u * quarter) << 16) + b * P::kBN;
            float* stg = staging + (warp - 2u) * (32u * 33u);
            if (a.epilogue == kGated) {
                // columns [128·part, +128): 64 gate then the same outputs' 64 up
#pragma unroll 1
                for (uint32_t h = 0; h < 2u; ++h) {
                    float g[32], u[32];
                    tmem_ld32(taddr + 128u * part + 32u * h, g);
                    tmem_ld32(taddr + 128u * part + 64u + 32u * h, u);
#pragma unroll
                    for (uint32_t j = 0; j < 32u; ++j) g[j] = activate(a.activation, g[j]) * u[j];
#pragma unroll
                    for (uint32_t j = 0; j < 32u; ++j) stg[lane * 33u + j] = g[j];
                    __syncwarp();
                    const uint32_t o = n0 / 2u + 64u * part + 32u * h + lane;
                    if (o < a.member[0].rows) {
                        const size_t at = static_cast<size_t>(t0) * a.out_stride[0] + a.member[0].out_offset + o;
                        float* dst = a.out[0] + at;
                        __half* dst16 = a.out16 ? static_cast<__half*>(a.out16) + at : nullptr;
                        for (uint32_t r = 0; r < 32u && t0 + r < a.tokens; ++r) {
                            const float v = stg[r * 33u + lane];
                            dst[static_cast<size_t>(r) * a.out_stride[0]] = v;
                            if (dst16) dst16[static_cast<size_t>(r) * a.out_stride[0]] = __float2half_rn(v);
                        }
                    }
                    __syncwarp();
                }
            } else {
#pragma unroll 1
                for (uint32_t c0 = 128u * part; c0 < 128u * part + 128u; c0 += 32u) {
                    float v[32];
                    tmem_ld32(taddr + c0, v);
                    store_block(a, t0, n0 + c0, v, slots, stg, lane);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
    }
    grid_dependents_launch();
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 2u * P::kBN);
    }
}

// The splits' partial sums added in order (split 0 first), then the
// epilogue. A thread an output of a token.
__global__ void dense_combine_kernel(const MatmulArgs a, uint32_t splits, const float* partials) {
    grid_dependency_wait();
    const uint32_t slots = dense_slot_count(a);
    const bool gated = a.epilogue == kGated;
    const uint32_t outputs = gated ? a.member[0].rows : slots;
    const size_t plane = static_cast<size_t>(a.tokens) * slots;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < a.tokens * outputs; i += gridDim.x * blockDim.x) {
        const uint32_t t = i / outputs, o = i % outputs;
        const uint32_t n = gated ? (o / 64u) * 128u + o % 64u : o;
        const float* p = partials + static_cast<size_t>(t) * slots + n;
        float v = p[0];
        for (uint32_t z = 1; z < splits; ++z) v += p[z * plane];
        if (gated) {
            float u = p[64];
            for (uint32_t z = 1; z < splits; ++z) u += p[z * plane + 64];
            put_gated(a, t, o, v, u);
        } else {
            put_slot(a, t, n, v);
        }
    }
    grid_dependents_launch();
}

template <uint32_t BN>
cudaError_t launch_dense(const MatmulArgs& a, const CUtensorMap& xmap, const CUtensorMap& wmap, uint32_t splits,
                         float* partials, cudaStream_t stream, bool pdl) {
    using S = Dense<BN>;
    auto kernel = dense_kernel<BN>;
    static bool configured = false;
    if (!configured) {
        const cudaError_t e =
            cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(S::kSmem));
        if (e != cudaSuccess) return e;
        configured = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((a.tokens + kBM - 1) / kBM, (dense_slot_count(a) + BN - 1) / BN, splits);
    cfg.blockDim = dim3(32 * S::kWarps);
    cfg.dynamicSmemBytes = S::kSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, a, xmap, wmap, splits, partials);
}

cudaError_t launch_persistent(const MatmulArgs& a, const CUtensorMap& xmap, const CUtensorMap& wmap, uint32_t ctas,
                              cudaStream_t stream, bool pdl) {
    static bool configured = false;
    if (!configured) {
        const cudaError_t e = cudaFuncSetAttribute(dense_persistent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(Persist::kSmem));
        if (e != cudaSuccess) return e;
        configured = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctas);
    cfg.blockDim = dim3(Persist::kThreads);
    cfg.dynamicSmemBytes = Persist::kSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, dense_persistent_kernel, a, xmap, wmap);
}

}  // namespace

uint64_t matmul_tensor_scratch_bytes(uint32_t tokens, uint32_t columns) {
    return (static_cast<uint64_t>(tokens) * columns * 2u + 255u) / 256u * 256u;
}

cudaError_t matmul_tensor(const MatmulArgs& a, cudaStream_t stream, bool pdl) {
    // 1. x to f16 in the scratch.
    if (cudaError_t e = launch_to_f16(a, stream, pdl); e != cudaSuccess) return e;
    // 2. The map of x16: [tokens][K] f16, boxes of 64 × 128.
    CUtensorMap map;
    if (cudaError_t e = encode_f16_map(&map, a.scratch, a.columns, a.tokens, kBM); e != cudaSuccess) return e;
    switch (a.format) {
        case kQ4_0: return launch_tensor<Q4_0>(a, map, stream, pdl);
        case kQ8_0: return launch_tensor<Q8_0>(a, map, stream, pdl);
        case kQ6_K: return launch_tensor<Q6_K>(a, map, stream, pdl);
        case kQ4_1: return launch_tensor<Q4_1>(a, map, stream, pdl);
        case kBF16: return launch_tensor<BF16>(a, map, stream, pdl);
        default: return cudaErrorInvalidValue;
    }
}


uint64_t matmul_dense_bytes(const MatmulArgs& a) {
    return static_cast<uint64_t>(dense_slot_count(a)) * a.columns * 2u;
}

cudaError_t matmul_densify(const MatmulArgs& a, void* dense, cudaStream_t stream) {
    const uint32_t slots = dense_slot_count(a);
    const uint32_t blocks = (slots + 7u) / 8u < 4096u ? (slots + 7u) / 8u : 4096u;
    uint4* d = static_cast<uint4*>(dense);
    switch (a.format) {
        case kQ4_0: densify_kernel<Q4_0><<<blocks, 256, 0, stream>>>(a, slots, d); break;
        case kQ8_0: densify_kernel<Q8_0><<<blocks, 256, 0, stream>>>(a, slots, d); break;
        case kQ6_K: densify_kernel<Q6_K><<<blocks, 256, 0, stream>>>(a, slots, d); break;
        case kQ4_1: densify_kernel<Q4_1><<<blocks, 256, 0, stream>>>(a, slots, d); break;
        case kBF16: densify_kernel<BF16><<<blocks, 256, 0, stream>>>(a, slots, d); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t matmul_dense(const MatmulArgs& a, int sms, cudaStream_t stream, bool pdl) {
    const uint32_t slots = dense_slot_count(a);
    const uint32_t sm = sms > 0 ? static_cast<uint32_t>(sms) : 148u;
    auto ceil_div = [](uint32_t n, uint32_t d) { return (n + d - 1u) / d; };
    // A wave or more of 128 × 256 tiles: the persistent form, a CTA an SM.
    // x as f16: given (a producer's copy), or rounded into the scratch
    const void* x16 = a.x16 ? a.x16 : a.scratch;
    const uint32_t wide_tiles = ceil_div(a.tokens, 128) * ceil_div(slots, 256);
    if (wide_tiles >= sm) {
        if (!a.x16)
            if (cudaError_t e = launch_to_f16(a, stream, pdl); e != cudaSuccess) return e;
        CUtensorMap xmap, wmap;
        if (cudaError_t e = encode_f16_map(&xmap, x16, a.columns, a.tokens, kBM); e != cudaSuccess) return e;
        if (cudaError_t e = encode_f16_map(&wmap, a.dense, a.columns, slots, Persist::kBN); e != cudaSuccess) return e;
        return launch_persistent(a, xmap, wmap, sm, stream, pdl);
    }
    // Fewer: 128 × 128 tiles, one a CTA, K split when they leave SMs idle.
    constexpr uint32_t bn = 128;
    const uint32_t tiles = ceil_div(a.tokens, 128) * ceil_div(slots, bn);
    // Split K where it shortens the product: the waves of CTAs a split
    // costs, over the splits, plus a sixth of an unsplit wave for writing
    // and adding the partials (a second launch adds them in order); each
    // split at least 8 K blocks, their partials where the scratch has room
    // after x16.
    const uint32_t kblocks = ceil_div(a.columns, kBK);
    const uint64_t x16_bytes = matmul_tensor_scratch_bytes(a.tokens, a.columns);
    uint32_t splits = 1;
    double best = static_cast<double>(ceil_div(tiles, sm));
    for (uint32_t z = 2; z <= 8u && kblocks / z >= 8u; ++z) {
        if (x16_bytes + static_cast<uint64_t>(z) * a.tokens * slots * 4u > a.scratch_bytes) break;
        const double cost = static_cast<double>(ceil_div(tiles * z, sm)) / z + 1.0 / 6.0;
        if (cost < best - 1e-9) {
            best = cost;
            splits = z;
        }
    }
    float* partials = splits > 1u ? reinterpret_cast<float*>(static_cast<uint8_t*>(a.scratch) + x16_bytes) : nullptr;

    if (!a.x16)
        if (cudaError_t e = launch_to_f16(a, stream, pdl); e != cudaSuccess) return e;
    CUtensorMap xmap, wmap;
    if (cudaError_t e = encode_f16_map(&xmap, x16, a.columns, a.tokens, kBM); e != cudaSuccess) return e;
    if (cudaError_t e = encode_f16_map(&wmap, a.dense, a.columns, slots, bn); e != cudaSuccess) return e;
    cudaError_t e = launch_dense<bn>(a, xmap, wmap, splits, partials, stream, pdl);
    if (e != cudaSuccess || splits == 1u) return e;
    const uint32_t outputs = a.epilogue == kGated ? a.member[0].rows : slots;
    const uint64_t n = static_cast<uint64_t>(a.tokens) * outputs;
    const uint32_t blocks = static_cast<uint32_t>((n + 255u) / 256u < 4096u ? (n + 255u) / 256u : 4096u);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks);
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, dense_combine_kernel, a, splits, static_cast<const float*>(partials));
}

}  // namespace cb
