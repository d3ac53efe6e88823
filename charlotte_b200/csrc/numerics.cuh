// Device numerics shared by every kernel of the hot path.
//
// Charlotte's kernels (plainsight-systems/charlotte, src/core/kernels/*.wgsl)
// fix each output's order of operations so that a token's bits do not depend
// on how its step was shaped (src/core/kernels/matmul/matmul.h:34-50, 596-604).
// Where WGSL leaves a result to the implementation, this backend fixes one
// definition and states it here; the CPU oracle (test infrastructure) states
// the same one, so the CUDA path and the oracle agree bit for bit:
//   dot4(a,b)       fmaf(a3,b3, fmaf(a2,b2, fmaf(a1,b1, a0*b0)))
//   inverseSqrt(v)  1.0f / sqrtf(v)   — correctly rounded division and sqrt
//   x*y + z*w       fmaf(x, y, z*w)
//   acc += p*v      fmaf(p, v, acc)
//   e^x (x <= 0)    Cody–Waite + Taylor to r^6 (matmul.wgsl:169-182)
//   2^x (x <= 0)    nearest-integer split + Taylor to degree 7 of e^(r ln 2)
//   sin, cos        Cody–Waite by pi/2 + Taylor to r^9 / r^10
//   ldexp(p, k)     multiplies by exact powers of two
// The library is compiled with --fmad=false, so only the explicit fmaf()
// calls below fuse; division and sqrt keep IEEE rounding (no fast-math).
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

namespace cb {

__device__ __forceinline__ float fp16_bits_to_f32(uint16_t h) {
    return __half2float(__ushort_as_half(h));   // exact, subnormals kept
}

// Saturate to +-65,504, then round to nearest even (f16_pack.wgsl:9-15).
__device__ __forceinline__ uint16_t f32_to_f16_sat(float v) {
    v = fminf(fmaxf(v, -65504.0f), 65504.0f);
    return __half_as_ushort(__float2half_rn(v));
}

__device__ __forceinline__ float scale2(float p, int k) {
    while (k < -126) { p = p * 0x1p-64f; k += 64; }
    while (k > 127) { p = p * 0x1p64f; k -= 64; }
    return p * __uint_as_float(static_cast<uint32_t>(k + 127) << 23);
}

// e^x for x <= 0 (matmul.wgsl:169-182).
__device__ __forceinline__ float exp_nonpositive(float x) {
    float xc = fmaxf(x, -100.0f);
    float k = floorf(fmaf(xc, 1.4426950408889634f, 0.5f));
    float r = fmaf(k, -0.693145751953125f, xc);
    r = fmaf(k, -1.4286068203094172e-06f, r);
    float p = 1.0f / 720.0f;
    p = fmaf(p, r, 1.0f / 120.0f);
    p = fmaf(p, r, 1.0f / 24.0f);
    p = fmaf(p, r, 1.0f / 6.0f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    return scale2(p, static_cast<int>(k));
}

enum Activation : int { kSiLU = 0, kGeluTanh = 1, kSigmoid = 2 };

// matmul.wgsl:189-205.
__device__ __forceinline__ float activate(int activation, float g) {
    if (activation == kSiLU) {
        float e = exp_nonpositive(-fabsf(g));
        float r = 1.0f / (1.0f + e);
        return g * (g >= 0.0f ? r : e * r);
    }
    if (activation == kSigmoid) {
        float e = exp_nonpositive(-fabsf(g));
        float r = 1.0f / (1.0f + e);
        return g >= 0.0f ? r : e * r;
    }
    float z = 0.7978845608028654f * fmaf(0.044715f * g * g, g, g);
    float e = exp_nonpositive(-2.0f * fabsf(z));
    float sgn = z > 0.0f ? 1.0f : (z < 0.0f ? -1.0f : 0.0f);
    float t = sgn * ((1.0f - e) * (1.0f / (1.0f + e)));
    float half_g = 0.5f * g;
    return fmaf(half_g, t, half_g);
}

// 2^x for x <= 0: x = k + r, r in [-1/2, 1/2]; e^(r ln 2) by Taylor to
// degree 7 in Horner form; then 2^k.
__device__ __forceinline__ float exp2_np(float x) {
    float xc = fmaxf(x, -160.0f);
    float k = floorf(xc + 0.5f);
    float r = xc - k;
    float t = r * 0.693147182f;
    float p = 1.0f / 5040.0f;
    p = fmaf(p, t, 1.0f / 720.0f);
    p = fmaf(p, t, 1.0f / 120.0f);
    p = fmaf(p, t, 1.0f / 24.0f);
    p = fmaf(p, t, 1.0f / 6.0f);
    p = fmaf(p, t, 0.5f);
    p = fmaf(p, t, 1.0f);
    p = fmaf(p, t, 1.0f);
    return scale2(p, static_cast<int>(k));
}

// sin and cos of an angle in [-pi, pi] (Cody–Waite by pi/2, Taylor series).
__device__ __forceinline__ void sincos_turn(float angle, float* s_out, float* c_out) {
    float q = rintf(angle * 0.636619772f);
    float r = fmaf(q, -1.57079625f, angle);
    r = fmaf(q, -7.54978942e-08f, r);
    float r2 = r * r;
    float ps = -1.0f / 39916800.0f;
    ps = fmaf(ps, r2, 1.0f / 362880.0f);
    ps = fmaf(ps, r2, -1.0f / 5040.0f);
    ps = fmaf(ps, r2, 1.0f / 120.0f);
    ps = fmaf(ps, r2, -1.0f / 6.0f);
    float s = fmaf(ps * r2, r, r);
    float pc = 1.0f / 3628800.0f;
    pc = fmaf(pc, r2, -1.0f / 40320.0f);
    pc = fmaf(pc, r2, 1.0f / 720.0f);
    pc = fmaf(pc, r2, -1.0f / 24.0f);
    pc = fmaf(pc, r2, 0.5f);
    float c = fmaf(-pc, r2, 1.0f);
    switch (static_cast<int>(q) & 3) {
        case 0: *s_out = s; *c_out = c; break;
        case 1: *s_out = c; *c_out = -s; break;
        case 2: *s_out = -s; *c_out = -c; break;
        default: *s_out = -c; *c_out = s; break;
    }
}

__device__ __forceinline__ float dot4(float4 a, float4 b) {
    return fmaf(a.w, b.w, fmaf(a.z, b.z, fmaf(a.y, b.y, a.x * b.x)));
}

// topk.wgsl:28-52: an order-preserving key of a logit's bits.
__host__ __device__ __forceinline__ uint32_t key_of(uint32_t b) {
    if (b == 0x80000000u) b = 0u;
    if ((b & 0x7F800000u) == 0x7F800000u && (b & 0x007FFFFFu) != 0u) return 0xFFFFFFFFu;
    if (b & 0x80000000u) return ~b;
    return b | 0x80000000u;
}

__host__ __device__ __forceinline__ uint32_t bits_of(uint32_t key) {
    if (key == 0xFFFFFFFFu) return 0x7FC00000u;
    if (key & 0x80000000u) return key & 0x7FFFFFFFu;
    return ~key;
}

// ---- packed fp32 pairs (Blackwell f32x2) -------------------------------------
// Two independent IEEE single-precision operations a lane per instruction:
// each half rounds exactly as the scalar fmaf would.

__device__ __forceinline__ unsigned long long pack2(float lo, float hi) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}

__device__ __forceinline__ void unpack2(unsigned long long v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}

__device__ __forceinline__ unsigned long long fma2(unsigned long long a, unsigned long long b,
                                                   unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

}  // namespace cb
