// A C ABI over the reference's own CPU code for the pinned pieces — TEST
// INFRASTRUCTURE ONLY. Compiled by oracle/Makefile against the reference
// project's sources where they lie (its tests/support headers,
// src/core/formats/q6_k/q6_k_repack.cpp and the rope launcher
// src/core/kernels/rope/rope.cpp); the output lands in oracle/_ref/.
// The tests use it to pin oracle.c: every dequantized weight, f16 pack and
// Q6_K repack byte of the oracle must equal the reference's, the rope turns
// its launcher writes, and the draw its f64 reference makes.
#include <array>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <span>
#include <vector>

#include "core/formats/device_layout.h"
#include "core/formats/f16/f16.h"
#include "core/kernels/rope/rope.h"
#include "core/quant/q4_0.h"
#include "support/f16_reference.h"
#include "support/q4_0_reference.h"
#include "support/q4_1_reference.h"
#include "support/q6_k_reference.h"
#include "support/q8_0_reference.h"
#include "support/sampler_reference.h"

namespace {
template <typename F>
int copy_out(F&& f, const std::uint8_t* data, std::size_t bytes, float* out) {
    const std::vector<float> v = f(std::span<const std::uint8_t>(data, bytes));
    std::memcpy(out, v.data(), v.size() * sizeof(float));
    return static_cast<int>(v.size());
}
}  // namespace

extern "C" {

// tests/support/q4_0_reference.h:25
int ref_dequant_q4_0(const std::uint8_t* data, std::size_t bytes, float* out) {
    return copy_out(bllm::test::dequantize_q4_0, data, bytes, out);
}
// tests/support/q8_0_reference.h:15
int ref_dequant_q8_0(const std::uint8_t* data, std::size_t bytes, float* out) {
    return copy_out(bllm::test::dequantize_q8_0, data, bytes, out);
}
// tests/support/q6_k_reference.h:17
int ref_dequant_q6_k(const std::uint8_t* data, std::size_t bytes, float* out) {
    return copy_out(bllm::test::dequantize_q6_k, data, bytes, out);
}
// tests/support/q4_1_reference.h:25: both evaluations it accepts, the
// multiply-add fused (one rounding) and rounded twice.
int ref_dequant_q4_1_fused(const std::uint8_t* data, std::size_t bytes, float* out) {
    return copy_out([](std::span<const std::uint8_t> s) { return bllm::test::dequantize_q4_1(s).fused; }, data,
                    bytes, out);
}
int ref_dequant_q4_1_rounded(const std::uint8_t* data, std::size_t bytes, float* out) {
    return copy_out([](std::span<const std::uint8_t> s) { return bllm::test::dequantize_q4_1(s).rounded; }, data,
                    bytes, out);
}
// src/core/quant/q4_0.h:66
float ref_fp16_to_fp32(std::uint16_t h) { return bllm::quant::fp16_to_fp32(h); }
// tests/support/f16_reference.h:14
std::uint16_t ref_fp32_to_fp16_saturating(float f) { return bllm::test::fp32_to_fp16_saturating(f); }
// src/core/formats/q6_k/q6_k_repack.cpp:52, through the layout's pointer
// (device_layout.h:159) as upload calls it.
void ref_repack_q6_k(const std::uint8_t* blocks, std::size_t count, std::uint8_t* lo, std::uint8_t* hi,
                     std::uint8_t* scales, std::uint8_t* d) {
    const auto* bytes = reinterpret_cast<const std::byte*>(blocks);
    bllm::formats::kQ6_KLayout.repack(std::span<const std::byte>(bytes, count * 210),
                                      {reinterpret_cast<std::byte*>(lo), reinterpret_cast<std::byte*>(hi),
                                       reinterpret_cast<std::byte*>(scales), reinterpret_cast<std::byte*>(d)});
}
// tests/support/sampler_reference.h (Philox4x32-10)
void ref_philox(const std::uint32_t counter[4], std::uint32_t key0, std::uint32_t key1, std::uint32_t out[4]) {
    bllm::testing::Philox c{{counter[0], counter[1], counter[2], counter[3]}};
    const bllm::testing::Philox r = bllm::testing::philox4x32_10(c, key0, key1);
    for (int i = 0; i < 4; ++i) out[i] = r.words[i];
}

// tests/support/sampler_reference.h uniform(): the draw's uniform for a
// 64-bit seed (low word first) and a position.
float ref_uniform(std::uint32_t seed_lo, std::uint32_t seed_hi, std::uint32_t position) {
    return bllm::testing::uniform((std::uint64_t{seed_hi} << 32) | seed_lo, position);
}
// tests/support/sampler_reference.h reference_draw(): the index the draw
// chooses given u, in f64, and how near it came to another decision.
// candidates: 64 (logit, token) pairs, best first.
void ref_reference_draw(const float* logits, const std::uint32_t* tokens, std::uint32_t count, float temperature,
                        std::uint32_t top_k, float top_p, float min_p, double u, std::uint32_t* chosen,
                        double* margin) {
    std::vector<bllm::testing::Candidate> c(count);
    for (std::uint32_t i = 0; i < count; ++i) c[i] = {logits[i], tokens[i]};
    const bllm::policy::SamplingSettings s{temperature, top_k, top_p, min_p};
    const bllm::testing::Reference r = bllm::testing::reference_draw(c, s, u);
    *chosen = static_cast<std::uint32_t>(r.chosen);
    *margin = r.margin;
}
// src/core/kernels/rope/rope.cpp:76-87 constants_of, through rope_launch,
// read back as tests/kernels_rope_test.cpp:48 reads it: the 256 turns at
// offset 16 of the launch's 1,040 bytes of constants.
int ref_rope_turns(float base, std::uint32_t head_dim, float* turns) {
    using namespace bllm;
    const model::LayerDescription layer{4, 1, head_dim, 3072, 40960, base, {}};
    const residency::BufferRange q{residency::BufferIndex{3}, 0, 100}, k{residency::BufferIndex{4}, 0, 200},
        v{residency::BufferIndex{5}, 0, 300};
    const residency::PlannedCacheLayer cache{{residency::BufferIndex{6}, 512, 4096},
                                             {residency::BufferIndex{6}, 4608, 4096}, 4608};
    const kernels::Launch l = kernels::rope_launch(
        {layer, model::RotaryPairing::Halves, nullptr, nullptr, nullptr, 1e-6f, q, k, v, cache, &formats::kF16});
    if (l.constants.size() != 1040) return -1;
    std::memcpy(turns, l.constants.data() + 16, 256 * sizeof(float));
    return 0;
}
}
