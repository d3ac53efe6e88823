// The device layout of a weight piece, made on the host from the file's
// stored blocks (plainsight-systems/charlotte, src/core/formats/
// device_layout.h:121-136; the Q6_K repack's placement is the one
// src/core/formats/q6_k/q6_k.h:9-21 states). What the reference's
// PieceWriter (src/core/residency/piece_writer.h) writes into a WebGPU
// buffer, this writes into host memory for one cudaMemcpy.
//
// Streams, each over every block in order: Q4_0 codes (16 B) then scales
// (2 B); Q8_0 codes (32 B) then scales; Q6_K, per super-block, group k's
// low nibbles at 16k (byte j: weight j's nibble low, weight j+16's high),
// its high bit pairs at 8k (byte m: weights m, m+8, m+16, m+24 from bit 0
// up), then the 16 scales and d as stored. The piece is padded to 16 bytes.
#include <cstdint>
#include <cstring>

#include "api_common.h"
#include "charlotte_b200.h"

namespace {

uint32_t block_bytes(uint32_t format) {
    switch (format) {
        case CB_F32: return 4;
        case CB_F16: return 2;
        case CB_Q4_0: return 18;
        case CB_Q4_1: return 20;
        case CB_BF16: return 2;
        case CB_Q8_0: return 34;
        case CB_Q6_K: return 210;
        default: return 0;
    }
}

// ggml's block_q6_K stores weight l of group k = 4h + r (half h, run r)
// with its low nibble as nibble r/2 of ql[64h + 32(r%2) + l] and its high
// pair as bits 2r..2r+1 of qh[32h + l].
void repack_q6_k(const uint8_t* blk, uint8_t* lo, uint8_t* hi) {
    std::memset(lo, 0, 128);
    std::memset(hi, 0, 64);
    for (int k = 0; k < 8; ++k) {
        const int h = k / 4, r = k % 4;
        const uint8_t* ql = blk + 64 * h + 32 * (r % 2);
        const uint8_t* qh = blk + 128 + 32 * h;
        for (int l = 0; l < 32; ++l) {
            const uint8_t nib = static_cast<uint8_t>((ql[l] >> (4 * (r / 2))) & 0xF);
            const uint8_t pair = static_cast<uint8_t>((qh[l] >> (2 * r)) & 3);
            lo[16 * k + l % 16] |= static_cast<uint8_t>(nib << (4 * (l / 16)));
            hi[8 * k + l % 8] |= static_cast<uint8_t>(pair << (2 * (l / 8)));
        }
    }
}

}  // namespace

extern "C" {

size_t cb_piece_bytes(uint32_t format, uint64_t blocks) {
    const uint64_t stored = blocks * block_bytes(format);
    return static_cast<size_t>((stored + 15u) & ~uint64_t{15});
}

int cb_piece_from_stored(uint32_t format, const void* stored_host, uint64_t blocks, void* piece_host) {
    if (!stored_host || !piece_host) return cb::fail(CB_ERROR_INVALID, "cb_piece_from_stored: null argument");
    if (block_bytes(format) == 0) return cb::fail(CB_ERROR_INVALID, "cb_piece_from_stored: format %u", format);
    const auto* st = static_cast<const uint8_t*>(stored_host);
    auto* out = static_cast<uint8_t*>(piece_host);
    std::memset(out, 0, cb_piece_bytes(format, blocks));
    switch (format) {
        case CB_Q4_0:
        case CB_Q8_0: {
            const uint32_t bb = block_bytes(format), cb = bb - 2;
            for (uint64_t b = 0; b < blocks; ++b) {
                std::memcpy(out + cb * b, st + bb * b + 2, cb);
                std::memcpy(out + cb * blocks + 2 * b, st + bb * b, 2);
            }
            return CB_OK;
        }
        case CB_Q4_1:   // codes, then each block's (d, m) word (device_layout.h:122)
            for (uint64_t b = 0; b < blocks; ++b) {
                std::memcpy(out + 16 * b, st + 20 * b + 4, 16);
                std::memcpy(out + 16 * blocks + 4 * b, st + 20 * b, 4);
            }
            return CB_OK;
        case CB_Q6_K:
            for (uint64_t b = 0; b < blocks; ++b) {
                const uint8_t* blk = st + 210 * b;
                repack_q6_k(blk, out + 128 * b, out + 128 * blocks + 64 * b);
                std::memcpy(out + 192 * blocks + 16 * b, blk + 192, 16);
                std::memcpy(out + 208 * blocks + 2 * b, blk + 208, 2);
            }
            return CB_OK;
        default:
            std::memcpy(out, st, blocks * block_bytes(format));
            return CB_OK;
    }
}

}  // extern "C"
