// A C ABI over the reference's own CPU code for the pinned pieces — TEST
// INFRASTRUCTURE ONLY. Compiled by oracle/Makefile against the reference
// project's sources where they lie (its tests/support headers and
// src/core/formats/q6_k/q6_k_repack.cpp); the output lands in oracle/_ref/.
// The tests use it to pin oracle.c: every dequantized weight, f16 pack and
// Q6_K repack byte of the oracle must equal the reference's.
#include <array>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <span>
#include <vector>

#include "core/formats/device_layout.h"
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
}
