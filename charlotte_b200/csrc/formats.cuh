// Weight formats on the device: Q4_0, Q8_0 and repacked Q6_K, read from the
// reference's device layout (plainsight-systems/charlotte,
// src/core/formats/device_layout.h:121-136): a piece holds every block's
// first field, then every block's next field — Q4_0 codes (16 B a block) then
// fp16 scales; Q8_0 codes (32 B) then scales; Q6_K low nibbles (128 B a
// super-block), high bit pairs (64 B), int8 scales (16 B), fp16 d (2 B),
// repacked at upload as src/core/formats/q6_k/q6_k.h:9-21 describes.
//
// Decoding is exact: every weight equals the format's unpack (q4_0.wgsl:6,
// q8_0.wgsl:6, q6_k.wgsl:13) bit for bit, computed in the load path, never
// written back expanded. Each weight is one fused multiply-add of a "magic"
// float: the code's bits OR'd into the mantissa of 1.0 give m = 1 + q·2^(j−23)
// exactly, and
//     w = fma(m, S, C),  S = s·2^(23−j),  C = −(S + z·s)
// equals (q − z)·s before rounding, where s is the block's scale and z its
// zero point; S and C are exact in binary32 (j is chosen so that C's
// significand fits), so the single rounding of the fma is the rounding of
// the reference's (q − z)·s. For Q4_0 and Q8_0 that product is exact; for
// Q6_K it is the reference's one rounding of (d·sc)·(q − 32). Two rows'
// weights may be decoded by one paired fma (__ffma2_rn: two independent
// fmas, each rounded once) from their constants as pairs (consts2): the
// same bits as two scalar fmas.
#pragma once

#include <cstdint>
#include <utility>

#include "numerics.cuh"

namespace cb {

enum Format : uint32_t { kF32 = 0, kF16 = 1, kQ4_0 = 2, kQ4_1 = 3, kQ8_0 = 8, kQ6_K = 14, kBF16 = 30 };

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    return __byte_perm(a, b, sel);
}

__device__ __forceinline__ float2 neg2(float2 v) { return make_float2(-v.x, -v.y); }

// Every format gives weight k of a group as weight<k>(f, consts) and the
// same weight of two rows at once as weight2<k>(a, b, consts2) (a paired
// fma rounds each half once: the bits of weight<k> on each row). The
// magic-float formats decode with one fma: w = fma(m, S, C).
template <typename F>
struct MagicDecode {
    template <int k, typename C>
    __device__ __forceinline__ static float weight(const F& f, const C& c) {
        return fmaf(__uint_as_float(f.template magic<k>()), F::template S<k>(c), F::template C<k>(c));
    }
    template <int k, typename C2>
    __device__ __forceinline__ static float2 weight2(const F& a, const F& b, const C2& c) {
        const float2 m = make_float2(__uint_as_float(a.template magic<k>()), __uint_as_float(b.template magic<k>()));
        return __ffma2_rn(m, F::template S2<k>(c), F::template C2<k>(c));
    }
};

// A 32-weight block of 4-bit codes (Q4_0, Q4_1): weight k is byte k % 16's
// low nibble for k < 16, its high nibble after. nibble_magic<k> moves the
// nibble into the mantissa of 1.0 at bit j = nibble_j<k>() (8, 12 or 16):
// the float 1 + q·2^(j−23), exactly.
template <int k>
__device__ __forceinline__ uint32_t nibble_magic(const uint4& codes) {
    constexpr int i = k % 4, w = (k % 16) / 4, h = k / 16;
    constexpr int pos = 8 * i + 4 * h;
    const uint32_t c = w == 0 ? codes.x : (w == 1 ? codes.y : (w == 2 ? codes.z : codes.w));
    if constexpr (pos >= 8 && pos <= 16) return (c & (0xFu << pos)) | 0x3F800000u;
    else if constexpr (pos >= 20) return ((c >> 12) & (0xFu << (pos - 12))) | 0x3F800000u;
    else return ((c << 8) & (0xFu << (pos + 8))) | 0x3F800000u;
}
template <int k>
__host__ __device__ static constexpr int nibble_j() {
    constexpr int pos = 8 * (k % 4) + 4 * (k / 16);
    return pos >= 8 && pos <= 16 ? pos : (pos >= 20 ? pos - 12 : pos + 8);
}

// ---- Q4_0 -------------------------------------------------------------------
// Weight k of a block: byte k % 16 of its codes, low nibble for k < 16, high
// nibble after (q4_0.wgsl:11-16); value (q − 8)·d.
struct Q4_0 : MagicDecode<Q4_0> {
    static constexpr uint32_t kGroupsPerBlock = 1;
    static constexpr int kStreams = 2;
    __host__ __device__ static constexpr uint32_t block_stream(int s) { return s == 0 ? 16u : 2u; }   // codes, d
    uint4 codes;
    float d;

    // Group g of a row whose streams were staged at s[0..1].
    __device__ __forceinline__ void load(const uint8_t* const* s, uint32_t g) {
        codes = *reinterpret_cast<const uint4*>(s[0] + 16u * g);
        d = fp16_bits_to_f32(*reinterpret_cast<const uint16_t*>(s[1] + 2u * g));
    }
    __device__ __forceinline__ void zero() { codes = make_uint4(0, 0, 0, 0); d = 0.0f; }

    // Constants by nibble position j in {8, 12, 16}.
    struct Consts { float s8, s12, s16, c8, c12, c16; };
    __device__ __forceinline__ Consts consts() const {
        Consts c;
        c.s8 = d * 32768.0f;
        c.s12 = d * 2048.0f;
        c.s16 = d * 128.0f;
        const float z = d * 8.0f;
        c.c8 = -(c.s8 + z);
        c.c12 = -(c.s12 + z);
        c.c16 = -(c.s16 + z);
        return c;
    }
    __device__ __forceinline__ uint32_t word(int w) const {
        return w == 0 ? codes.x : (w == 1 ? codes.y : (w == 2 ? codes.z : codes.w));
    }
    // The magic float of weight k (k a compile-time constant once unrolled),
    // and which constants (j) it takes.
    template <int k>
    __device__ __forceinline__ uint32_t magic() const { return nibble_magic<k>(codes); }
    template <int k>
    __host__ __device__ static constexpr int jpos() { return nibble_j<k>(); }
    template <int k>
    __device__ __forceinline__ static float S(const Consts& c) {
        constexpr int j = jpos<k>();
        return j == 8 ? c.s8 : (j == 12 ? c.s12 : c.s16);
    }
    template <int k>
    __device__ __forceinline__ static float C(const Consts& c) {
        constexpr int j = jpos<k>();
        return j == 8 ? c.c8 : (j == 12 ? c.c12 : c.c16);
    }
    // Two rows' constants as pairs (row A, row B): consts() of each, the same
    // operations elementwise.
    struct Consts2 { float2 s8, s12, s16, c8, c12, c16; };
    __device__ __forceinline__ static Consts2 consts2(const Q4_0& A, const Q4_0& B) {
        const float2 d = make_float2(A.d, B.d);
        Consts2 c;
        c.s8 = __fmul2_rn(d, make_float2(32768.0f, 32768.0f));
        c.s12 = __fmul2_rn(d, make_float2(2048.0f, 2048.0f));
        c.s16 = __fmul2_rn(d, make_float2(128.0f, 128.0f));
        const float2 z = __fmul2_rn(d, make_float2(8.0f, 8.0f));
        c.c8 = neg2(__fadd2_rn(c.s8, z));
        c.c12 = neg2(__fadd2_rn(c.s12, z));
        c.c16 = neg2(__fadd2_rn(c.s16, z));
        return c;
    }
    template <int k>
    __device__ __forceinline__ static float2 S2(const Consts2& c) {
        constexpr int j = jpos<k>();
        return j == 8 ? c.s8 : (j == 12 ? c.s12 : c.s16);
    }
    template <int k>
    __device__ __forceinline__ static float2 C2(const Consts2& c) {
        constexpr int j = jpos<k>();
        return j == 8 ? c.c8 : (j == 12 ? c.c12 : c.c16);
    }
};

// ---- Q8_0 -------------------------------------------------------------------
// Weight k: signed byte k of the codes; value q·d (q8_0.wgsl:11-15). The
// byte, offset by 128, lies at mantissa bits 8..15 (j = 8).
struct Q8_0 : MagicDecode<Q8_0> {
    static constexpr uint32_t kGroupsPerBlock = 1;
    static constexpr int kStreams = 2;
    __host__ __device__ static constexpr uint32_t block_stream(int s) { return s == 0 ? 32u : 2u; }   // codes, d
    uint4 lo, hi;
    float d;

    __device__ __forceinline__ void load(const uint8_t* const* s, uint32_t g) {
        const uint4* p = reinterpret_cast<const uint4*>(s[0] + 32u * g);
        lo = p[0];
        hi = p[1];
        d = fp16_bits_to_f32(*reinterpret_cast<const uint16_t*>(s[1] + 2u * g));
        lo.x ^= 0x80808080u; lo.y ^= 0x80808080u; lo.z ^= 0x80808080u; lo.w ^= 0x80808080u;
        hi.x ^= 0x80808080u; hi.y ^= 0x80808080u; hi.z ^= 0x80808080u; hi.w ^= 0x80808080u;
    }
    __device__ __forceinline__ void zero() {
        lo = make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);
        hi = lo;
        d = 0.0f;
    }
    struct Consts { float s, c; };
    __device__ __forceinline__ Consts consts() const {
        Consts c;
        c.s = d * 32768.0f;
        c.c = -(c.s + d * 128.0f);
        return c;
    }
    __device__ __forceinline__ uint32_t word(int w) const {
        switch (w) {
            case 0: return lo.x; case 1: return lo.y; case 2: return lo.z; case 3: return lo.w;
            case 4: return hi.x; case 5: return hi.y; case 6: return hi.z; default: return hi.w;
        }
    }
    template <int k>
    __device__ __forceinline__ uint32_t magic() const {
        // bytes: [0x00, code byte k%4, 0x80, 0x3F] -> 0x3F800000 | (q + 128) << 8
        return prmt(word(k / 4), 0x3F800000u, 0x7604u | ((k % 4) << 4));
    }
    template <int k>
    __device__ __forceinline__ static float S(const Consts& c) { return c.s; }
    template <int k>
    __device__ __forceinline__ static float C(const Consts& c) { return c.c; }
    struct Consts2 { float2 s, c; };
    __device__ __forceinline__ static Consts2 consts2(const Q8_0& A, const Q8_0& B) {
        const float2 d = make_float2(A.d, B.d);
        Consts2 c;
        c.s = __fmul2_rn(d, make_float2(32768.0f, 32768.0f));
        c.c = neg2(__fadd2_rn(c.s, __fmul2_rn(d, make_float2(128.0f, 128.0f))));
        return c;
    }
    template <int k>
    __device__ __forceinline__ static float2 S2(const Consts2& c) { return c.s; }
    template <int k>
    __device__ __forceinline__ static float2 C2(const Consts2& c) { return c.c; }
};

// ---- Q6_K (repacked) ----------------------------------------------------------
// Group k of a super-block: 16 bytes of low nibbles (byte j: weight j's, then
// weight j+16's), 8 bytes of high pairs (byte m: weights m, m+8, m+16, m+24
// from bit 0 up), scales 2k and 2k+1 for weights 0..15 and 16..31, and the
// block's d; value (d·sc)·(q − 32) (q6_k.wgsl:13-42). q's six bits sit at
// mantissa bits 16..21 (j = 16).
struct Q6_K : MagicDecode<Q6_K> {
    static constexpr uint32_t kGroupsPerBlock = 8;
    static constexpr int kStreams = 4;
    __host__ __device__ static constexpr uint32_t block_stream(int s) {   // lo, hi, scales, d
        return s == 0 ? 128u : (s == 1 ? 64u : (s == 2 ? 16u : 2u));
    }
    uint32_t a[4], b[4];   // per low-nibble word: weights 4w+i (a) and 16+4w+i (b), 0x80|q per byte
    float s1, s2;          // d·sc for weights 0..15 and 16..31

    __device__ __forceinline__ void load(const uint8_t* const* s, uint32_t g) {
        const uint4 lo = *reinterpret_cast<const uint4*>(s[0] + 16u * g);
        const uint2 hi = *reinterpret_cast<const uint2*>(s[1] + 8u * g);
        const uint16_t sc = *reinterpret_cast<const uint16_t*>(s[2] + 2u * g);
        const float d = fp16_bits_to_f32(*reinterpret_cast<const uint16_t*>(s[3] + 2u * (g >> 3)));
        s1 = d * static_cast<float>(static_cast<int8_t>(sc & 0xFF));
        s2 = d * static_cast<float>(static_cast<int8_t>(sc >> 8));
        const uint32_t lw[4] = {lo.x, lo.y, lo.z, lo.w};
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const uint32_t h = (w & 1) ? hi.y : hi.x;
            const int s = 2 * (w / 2);
            a[w] = (lw[w] & 0x0F0F0F0Fu) | ((h << (4 - s)) & 0x30303030u) | 0x80808080u;
            b[w] = ((lw[w] >> 4) & 0x0F0F0F0Fu) | ((h >> s) & 0x30303030u) | 0x80808080u;
        }
    }
    __device__ __forceinline__ void zero() {
#pragma unroll
        for (int w = 0; w < 4; ++w) { a[w] = 0x80808080u; b[w] = 0x80808080u; }
        s1 = 0.0f; s2 = 0.0f;
    }
    struct Consts { float S1, S2, C1, C2; };
    __device__ __forceinline__ Consts consts() const {
        Consts c;
        c.S1 = s1 * 128.0f;
        c.S2 = s2 * 128.0f;
        c.C1 = s1 * -160.0f;
        c.C2 = s2 * -160.0f;
        return c;
    }
    template <int k>
    __device__ __forceinline__ uint32_t magic() const {
        constexpr int w = (k % 16) / 4, i = k % 4;
        const uint32_t src = k < 16 ? a[w] : b[w];
        // bytes: [0x00, 0x00, 0x80|q, 0x3F]
        return prmt(src, 0x3F000000u, 0x7054u | (i << 8));
    }
    template <int k>
    __device__ __forceinline__ static float S(const Consts& c) { return k < 16 ? c.S1 : c.S2; }
    template <int k>
    __device__ __forceinline__ static float C(const Consts& c) { return k < 16 ? c.C1 : c.C2; }
    struct Consts2 { float2 S1, S2, C1, C2; };
    __device__ __forceinline__ static Consts2 consts2(const Q6_K& A, const Q6_K& B) {
        const float2 s1 = make_float2(A.s1, B.s1), s2 = make_float2(A.s2, B.s2);
        Consts2 c;
        c.S1 = __fmul2_rn(s1, make_float2(128.0f, 128.0f));
        c.S2 = __fmul2_rn(s2, make_float2(128.0f, 128.0f));
        c.C1 = __fmul2_rn(s1, make_float2(-160.0f, -160.0f));
        c.C2 = __fmul2_rn(s2, make_float2(-160.0f, -160.0f));
        return c;
    }
    template <int k>
    __device__ __forceinline__ static float2 S2(const Consts2& c) { return k < 16 ? c.S1 : c.S2; }
    template <int k>
    __device__ __forceinline__ static float2 C2(const Consts2& c) { return k < 16 ? c.C1 : c.C2; }
};

// ---- Q4_1 -------------------------------------------------------------------
// Weight k: the nibble of Q4_0's place, value q·d + m (q4_1.wgsl:6-20), the
// multiply and add fused, rounded once — one of the two evaluations the
// reference accepts (tests/support/q4_1_reference.h:13-21). The device
// layout holds every block's 16 code bytes, then every block's (d, m) word,
// d in its low half. q comes out of the magic float exactly (one fma by
// ±2^(23−j)), then w = fma(q, d, m).
struct Q4_1 {
    static constexpr uint32_t kGroupsPerBlock = 1;
    static constexpr int kStreams = 2;
    __host__ __device__ static constexpr uint32_t block_stream(int s) { return s == 0 ? 16u : 4u; }   // codes, (d, m)
    uint4 codes;
    float d, m;

    __device__ __forceinline__ void load(const uint8_t* const* s, uint32_t g) {
        codes = *reinterpret_cast<const uint4*>(s[0] + 16u * g);
        const uint32_t dm = *reinterpret_cast<const uint32_t*>(s[1] + 4u * g);
        d = fp16_bits_to_f32(static_cast<uint16_t>(dm & 0xFFFFu));
        m = fp16_bits_to_f32(static_cast<uint16_t>(dm >> 16));
    }
    __device__ __forceinline__ void zero() { codes = make_uint4(0, 0, 0, 0); d = 0.0f; m = 0.0f; }
    struct Consts { float d, m; };
    __device__ __forceinline__ Consts consts() const { return Consts{d, m}; }
    struct Consts2 { float2 d, m; };
    __device__ __forceinline__ static Consts2 consts2(const Q4_1& A, const Q4_1& B) {
        return Consts2{make_float2(A.d, B.d), make_float2(A.m, B.m)};
    }
    // 2^(23−j) for weight k (k < 32; larger k, instantiated but never run
    // by kernels that decode half a group at a time, take 1).
    template <int k>
    __host__ __device__ static constexpr float unit() {
        return nibble_j<k>() <= 23 ? static_cast<float>(1u << (nibble_j<k>() <= 23 ? 23 - nibble_j<k>() : 0)) : 1.0f;
    }
    template <int k>
    __device__ __forceinline__ static float code(const Q4_1& f) {
        constexpr float P = unit<k>();
        return fmaf(__uint_as_float(nibble_magic<k>(f.codes)), P, -P);
    }
    template <int k>
    __device__ __forceinline__ static float weight(const Q4_1& f, const Consts& c) {
        return fmaf(code<k>(f), c.d, c.m);
    }
    template <int k>
    __device__ __forceinline__ static float2 weight2(const Q4_1& a, const Q4_1& b, const Consts2& c) {
        constexpr float P = unit<k>();
        const float2 mg = make_float2(__uint_as_float(nibble_magic<k>(a.codes)), __uint_as_float(nibble_magic<k>(b.codes)));
        const float2 q = __ffma2_rn(mg, make_float2(P, P), make_float2(-P, -P));
        return __ffma2_rn(q, c.d, c.m);
    }
};

// ---- BF16 -------------------------------------------------------------------
// Each value is the top half of an f32 (bf16.wgsl:1-20): nothing computed.
// Groups of 32 values, 64 bytes (the bandwidth and stream accounting counts
// such a group as a block); value k is half k % 2 of word k / 2, the lower
// half first.
struct BF16 {
    static constexpr uint32_t kGroupsPerBlock = 1;
    static constexpr int kStreams = 1;
    __host__ __device__ static constexpr uint32_t block_stream(int) { return 64u; }
    uint4 v[4];

    __device__ __forceinline__ void load(const uint8_t* const* s, uint32_t g) {
        const uint4* p = reinterpret_cast<const uint4*>(s[0] + 64u * g);
        v[0] = p[0]; v[1] = p[1]; v[2] = p[2]; v[3] = p[3];
    }
    __device__ __forceinline__ void zero() {
        v[0] = v[1] = v[2] = v[3] = make_uint4(0, 0, 0, 0);
    }
    struct Consts {};
    __device__ __forceinline__ Consts consts() const { return Consts{}; }
    struct Consts2 {};
    __device__ __forceinline__ static Consts2 consts2(const BF16&, const BF16&) { return Consts2{}; }
    template <int k>
    __device__ __forceinline__ static float weight(const BF16& f, const Consts&) {
        const uint4& q = f.v[k / 8];
        constexpr int w = (k % 8) / 2;
        const uint32_t word = w == 0 ? q.x : (w == 1 ? q.y : (w == 2 ? q.z : q.w));
        return __uint_as_float(k % 2 == 0 ? word << 16 : word & 0xFFFF0000u);
    }
    template <int k>
    __device__ __forceinline__ static float2 weight2(const BF16& a, const BF16& b, const Consts2&) {
        return make_float2(weight<k>(a, Consts{}), weight<k>(b, Consts{}));
    }
};

// A row's streams: stream s of row r of a piece of `nb` blocks starts at
// base(s) + r·row_bytes(s) and is row_bytes(s) long (device_layout.h's
// streams, each over every block in order).
template <typename F>
struct RowStreams {
    __host__ __device__ static uint64_t base(int s, uint32_t nb) {
        uint64_t b = 0;
        for (int t = 0; t < s; ++t) b += static_cast<uint64_t>(F::block_stream(t)) * nb;
        return b;
    }
    __host__ __device__ static uint32_t row_bytes(int s, uint32_t G) {
        return G / F::kGroupsPerBlock * F::block_stream(s);
    }
    // Bytes of stream s's slot in a staged row: 16-aligned, with room for a
    // copy rounded out to 16-byte bounds when rows are not 16-byte multiples.
    __host__ __device__ static uint32_t slot(int s, uint32_t G) {
        const uint32_t n = row_bytes(s, G);
        return (n + 15u) / 16u * 16u + (n % 16u ? 16u : 0u);
    }
    __host__ __device__ static uint32_t row_stage(uint32_t G) {
        uint32_t t = 0;
        for (int s = 0; s < F::kStreams; ++s) t += slot(s, G);
        return t;
    }
};

// Bytes of weight data a 32-weight group occupies, for bandwidth accounting.
__host__ __device__ constexpr double group_bytes(uint32_t format) {
    return format == kQ4_0 ? 18.0
         : format == kQ4_1 ? 20.0
         : format == kQ8_0 ? 34.0
         : format == kQ6_K ? 210.0 / 8.0
         : format == kBF16 ? 64.0 : 0.0;
}

}  // namespace cb
