"""Pins the CPU oracle before it is trusted: against the reference's own CPU
code compiled from its sources (oracle/_ref: its tests/support dequantizers,
f16 conversions, Philox, and its Q6_K repack), and against the known answers
its tests state (tests/quant_q4_0_test.cpp, tests/sampler_test.cpp,
tests/formats_q6_k_repack_test.cpp). No GPU."""
import ctypes
import struct

import numpy as np
import pytest

import oracle as O
from charlotte_b200 import synth

REF = O.ref()
needs_ref = pytest.mark.skipif(REF is None, reason="oracle/_ref not built (the reference sources are absent)")


def _ref_dequant(fmt, stored):
    out = np.empty(stored.size // O.BLOCK_BYTES[fmt] * O.BLOCK_WEIGHTS[fmt], np.float32)
    fn = {O.Q4_0: REF.ref_dequant_q4_0, O.Q8_0: REF.ref_dequant_q8_0, O.Q6_K: REF.ref_dequant_q6_k,
          O.Q4_1: REF.ref_dequant_q4_1_fused}[fmt]
    fn(O.ptr(stored, ctypes.c_uint8), stored.size, O.ptr(out, ctypes.c_float))
    return out


@needs_ref
@pytest.mark.parametrize("fmt", [O.Q4_0, O.Q4_1, O.Q8_0, O.Q6_K])
@pytest.mark.parametrize("gen", ["random_bytes", "config"])
def test_dequant_matches_reference_bit_for_bit(fmt, gen):
    rng = np.random.default_rng(fmt * 7 + len(gen))
    n = 257
    stored = (synth.random_bytes_blocks(rng, fmt, n) if gen == "random_bytes"
              else synth.blocks(rng, fmt, n * O.BLOCK_WEIGHTS[fmt] // 32, 32))
    ours = O.dequant_stored(fmt, stored)
    theirs = _ref_dequant(fmt, stored)
    assert np.array_equal(ours, theirs)   # zeros compare by value, as format.h states


@needs_ref
@pytest.mark.parametrize("fmt", [O.Q4_0, O.Q4_1, O.Q8_0, O.Q6_K])
def test_unpack_from_device_layout_equals_reference_dequant(fmt):
    rng = np.random.default_rng(100 + fmt)
    n = 64
    stored = synth.random_bytes_blocks(rng, fmt, n)
    piece = O.to_piece(fmt, stored)
    groups = n * O.BLOCK_WEIGHTS[fmt] // 32
    got = np.concatenate([O.unpack(fmt, piece, n, g) for g in range(groups)])
    assert np.array_equal(got, _ref_dequant(fmt, stored))


@needs_ref
def test_q6_k_repack_matches_reference_repack():
    rng = np.random.default_rng(5)
    n = 33
    stored = synth.random_bytes_blocks(rng, O.Q6_K, n)
    lo, hi, sc, d = (np.zeros(n * w, np.uint8) for w in (128, 64, 16, 2))
    REF.ref_repack_q6_k(O.ptr(stored, ctypes.c_uint8), n, O.ptr(lo, ctypes.c_uint8), O.ptr(hi, ctypes.c_uint8),
                        O.ptr(sc, ctypes.c_uint8), O.ptr(d, ctypes.c_uint8))
    piece = O.to_piece(O.Q6_K, stored)
    assert np.array_equal(piece[: 210 * n], np.concatenate([lo, hi, sc, d]))
    assert np.array_equal(synth.to_piece(O.Q6_K, stored), piece)


@needs_ref
def test_q4_1_is_one_of_the_reference_evaluations():
    """The reference accepts a Q4_1 weight rounded once (fused) or twice
    (tests/support/q4_1_reference.h:13-21); this build takes the fused one:
    it equals the reference's fused value everywhere, and over typical blocks
    most weights agree with the twice-rounded value too."""
    rng = np.random.default_rng(41)
    stored = synth.blocks(rng, O.Q4_1, 64, 256)
    n = stored.size // 20
    fused, rounded = (np.empty(n * 32, np.float32) for _ in range(2))
    REF.ref_dequant_q4_1_fused(O.ptr(stored, ctypes.c_uint8), stored.size, O.ptr(fused, ctypes.c_float))
    REF.ref_dequant_q4_1_rounded(O.ptr(stored, ctypes.c_uint8), stored.size, O.ptr(rounded, ctypes.c_float))
    ours = O.dequant_stored(O.Q4_1, stored)
    assert np.array_equal(ours, fused)
    assert np.mean(ours == rounded) > 0.5


def test_bf16_is_the_top_half_of_an_f32():
    rng = np.random.default_rng(42)
    stored = synth.random_bytes_blocks(rng, O.BF16, 999)
    want = (stored.view(np.uint16).astype(np.uint32) << 16).view(np.float32)
    assert np.array_equal(O.dequant_stored(O.BF16, stored), want)
    piece = O.to_piece(O.BF16, stored)
    got = np.concatenate([O.unpack(O.BF16, piece, 999, g) for g in range(999 // 32)])
    assert np.array_equal(got, want[: got.size])


@pytest.mark.parametrize("fmt", [O.Q4_0, O.Q4_1, O.Q8_0, O.Q6_K, O.BF16])
def test_synth_device_layout_equals_oracle_layout(fmt):
    rng = np.random.default_rng(9)
    stored = synth.random_bytes_blocks(rng, fmt, 40)
    assert np.array_equal(synth.to_piece(fmt, stored), O.to_piece(fmt, stored))


@needs_ref
def test_fp16_conversions_match_reference():
    L = O.lib()
    for h in range(1 << 16):
        a, b = L.or_fp16_to_fp32(h), REF.ref_fp16_to_fp32(h)
        assert (np.isnan(a) and np.isnan(b)) or np.float32(a).view(np.uint32) == np.float32(b).view(np.uint32)
    rng = np.random.default_rng(3)
    xs = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s
                         for s in (1e-9, 1e-7, 1e-5, 1e-3, 1.0, 1e2, 6.5e4, 1e6)])
    xs = np.concatenate([xs, np.float32([65504, 65519, 65520, 70000, -65520, 2.0 ** -24, 2.0 ** -25, 0.0, -0.0])])
    for x in xs:
        assert L.or_fp32_to_fp16_sat(float(x)) == REF.ref_fp32_to_fp16_saturating(float(x))


def test_q4_0_known_answers():
    """tests/quant_q4_0_test.cpp: scale 1 gives nibble - 8; nibble 8 is zero;
    element 16 is the high nibble of byte 0; scale applies per block."""
    def block(scale_bits, nibbles):
        qs = bytes((nibbles[j] & 0xF) | ((nibbles[j + 16] & 0xF) << 4) for j in range(16))
        return np.frombuffer(struct.pack("<H", scale_bits) + qs, np.uint8)
    out = O.dequant_stored(O.Q4_0, block(0x3C00, [i % 16 for i in range(32)]))
    assert out.tolist() == [float(i % 16 - 8) for i in range(32)]
    assert not O.dequant_stored(O.Q4_0, block(0x4900, [8] * 32)).any()
    n = [8] * 32
    n[16] = 15
    out = O.dequant_stored(O.Q4_0, block(0x3C00, n))
    assert out[16] == 7.0 and out[0] == 0.0 and out[1] == 0.0 and out[8] == 0.0
    two = np.concatenate([block(0x3C00, [9] * 32), block(0x4000, [9] * 32)])
    out = O.dequant_stored(O.Q4_0, two)
    assert out[0] == 1.0 and out[32] == 2.0


def test_fp16_classes():
    """tests/quant_q4_0_test.cpp:41-65."""
    f = O.lib().or_fp16_to_fp32
    assert f(0x0000) == 0.0 and np.signbit(np.float32(f(0x8000)))
    assert f(0x3C00) == 1.0 and f(0xBC00) == -1.0 and f(0x7BFF) == 65504.0
    assert f(0x0001) == 2.0 ** -24 and f(0x0002) == 2.0 ** -23
    assert np.isinf(f(0x7C00)) and np.isnan(f(0x7E00))


def test_philox_random123_known_answers():
    """tests/sampler_test.cpp:15-31 (Random123's published vectors)."""
    cases = [
        ([0, 0, 0, 0], [0, 0], [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]),
        ([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2, [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]),
        ([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344], [0xA4093822, 0x299F31D0],
         [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]),
    ]
    for counter, key, want in cases:
        assert O.philox(counter, key).tolist() == want


def test_q6_k_repack_known_placement():
    """tests/formats_q6_k_repack_test.cpp:40-67: every weight's six bits where
    q6_k.h says, from where ggml's block_q6_K stores them."""
    rng = np.random.default_rng(11)
    st = synth.random_bytes_blocks(rng, O.Q6_K, 3).reshape(3, 210)
    piece = O.to_piece(O.Q6_K, st.reshape(-1))
    n = 3
    for b in range(n):
        lo = piece[128 * b: 128 * b + 128]
        hi = piece[128 * n + 64 * b: 128 * n + 64 * b + 64]
        for k in range(8):
            h, r = divmod(k, 4)
            for l in range(32):
                stored = ((st[b, 64 * h + 32 * (r % 2) + l] >> (4 * (r // 2))) & 0xF) | \
                         (((st[b, 128 + 32 * h + l] >> (2 * r)) & 3) << 4)
                rep = ((lo[16 * k + l % 16] >> (4 * (l // 16))) & 0xF) | (((hi[8 * k + l % 8] >> (2 * (l // 8))) & 3) << 4)
                assert stored == rep
        assert np.array_equal(piece[192 * n + 16 * b: 192 * n + 16 * b + 16], st[b, 192:208])
        assert np.array_equal(piece[208 * n + 2 * b: 208 * n + 2 * b + 2], st[b, 208:210])


def test_matmul_order_against_f64_bound():
    """matmul.h:'Accuracy': each output within gamma(2K)*sum|w x| of the f64 sum."""
    rng = np.random.default_rng(21)
    rows, K = 96, 3072
    st = synth.blocks(rng, O.Q4_0, rows, K)
    piece = O.to_piece(O.Q4_0, st)
    x = rng.standard_normal((2, K)).astype(np.float32)
    y = O.matmul(O.Q4_0, piece, rows * K // 32, rows, K, x)
    W = O.dequant_stored(O.Q4_0, st).reshape(rows, K).astype(np.float64)
    exact = x.astype(np.float64) @ W.T
    u = 2.0 ** -24
    gamma = 2 * K * u / (1 - 2 * K * u)
    bound = gamma * (np.abs(x.astype(np.float64)) @ np.abs(W).T)
    assert np.all(np.abs(y - exact) <= bound)


def test_sincos_against_libm():
    """The rotation's sine/cosine method stays within a few ulps of libm."""
    import math
    s = np.empty(1, np.float32)
    c = np.empty(1, np.float32)
    worst = 0.0
    for a in np.linspace(-math.pi, math.pi, 20001, dtype=np.float32):
        O.lib().or_sincos(float(a), O.ptr(s, ctypes.c_float), O.ptr(c, ctypes.c_float))
        worst = max(worst, abs(float(s[0]) - math.sin(float(a))), abs(float(c[0]) - math.cos(float(a))))
    assert worst < 4e-7


def test_exp2_and_exp_against_libm():
    import math
    worst2 = worst = 0.0
    # results in binary32's normal range (below it the result is subnormal)
    for x in np.linspace(-87.0, 0.0, 50001, dtype=np.float32):
        a = O.lib().or_exp2(float(x))
        e = 2.0 ** float(x)
        worst2 = max(worst2, abs(a - e) / e)
        b = O.lib().or_exp_nonpositive(float(x))
        e = math.exp(float(x))
        worst = max(worst, abs(b - e) / e)
    assert worst2 < 4e-7 and worst < 4e-7


# ---- the rope turns and the draw, against the reference's own code ----------

@needs_ref
@pytest.mark.parametrize("base", [1e6, 5e5, 1e4])
@pytest.mark.parametrize("d", [64, 128, 256, 512])
def test_rope_turns_equal_the_reference_launchers(base, d):
    """src/core/kernels/rope/rope.cpp:76-87 (constants_of), read back from the
    reference's rope_launch as tests/kernels_rope_test.cpp:48 reads it: the
    oracle's turns and the library's (cb_rope_turns, a host function) are
    the same bits, and the unused slots are zero."""
    import charlotte_b200 as cb
    ref = np.zeros(256, np.float32)
    REF.ref_rope_turns.argtypes = [ctypes.c_float, ctypes.c_uint32, ctypes.POINTER(ctypes.c_float)]
    assert REF.ref_rope_turns(base, d, O.ptr(ref, ctypes.c_float)) == 0
    assert not ref[d // 2:].any()
    assert np.array_equal(O.rope_turns(base, d).view(np.uint32), ref[: d // 2].view(np.uint32))
    assert np.array_equal(cb.rope_turns(base, d).view(np.uint32), ref[: d // 2].view(np.uint32))


def _candidates(seed):
    """64 candidates, best first, as the reference's draw test makes them
    (tests/gpu/draw_test.cpp:90-101): logits falling by up to 0.25 a step
    from 5, tokens below Qwen3's vocabulary."""
    state = np.uint32(seed)
    logit = np.float32(5.0)
    logits, tokens = [], []
    for _ in range(64):
        state = np.uint32((int(state) * 1664525 + 1013904223) & 0xFFFFFFFF)
        logit = np.float32(logit - np.float32(((int(state) >> 8) % 1000) / np.float32(4000.0)))
        logits.append(logit)
        tokens.append(((int(state) >> 4) % 151936))
    return np.array(logits, np.float32), np.array(tokens, np.uint32)


def _pairs(logits, tokens):
    pairs = np.empty(128, np.uint32)
    pairs[0::2] = logits.view(np.uint32)
    pairs[1::2] = tokens
    return pairs


def _ref_draw(logits, tokens, s, u):
    chosen = ctypes.c_uint32()
    margin = ctypes.c_double()
    REF.ref_reference_draw.argtypes = [ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_uint32),
                                       ctypes.c_uint32, ctypes.c_float, ctypes.c_uint32, ctypes.c_float,
                                       ctypes.c_float, ctypes.c_double, ctypes.POINTER(ctypes.c_uint32),
                                       ctypes.POINTER(ctypes.c_double)]
    REF.ref_reference_draw(O.ptr(logits, ctypes.c_float), O.ptr(tokens, ctypes.c_uint32), 64, s[0], s[1], s[2],
                           s[3], u, ctypes.byref(chosen), ctypes.byref(margin))
    return chosen.value, margin.value


def _ref_uniform(seed, position):
    REF.ref_uniform.restype = ctypes.c_float
    REF.ref_uniform.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32]
    return np.float32(REF.ref_uniform(seed & 0xFFFFFFFF, seed >> 32, position))


# (temperature, top_k, top_p, min_p): the reference's draw test's settings
DRAW_SETTINGS = [(0.8, 40, 0.95, 0.05), (0.6, 20, 0.95, 0.0), (1.0, 64, 0.95, 0.0), (1.5, 64, 1.0, 0.01),
                 (0.3, 8, 0.5, 0.2)]


@needs_ref
def test_draw_uniform_is_the_reference_philox_bit_for_bit():
    """tests/gpu/draw_test.cpp:104-125 on the oracle: a step of `tokens`
    from `position` draws with uniform(seed, position + tokens)."""
    logits, tokens = _candidates(1)
    pairs = _pairs(logits, tokens)
    for seed in (0, 1, 0x0123456789ABCDEF):
        for position in (0, 1, 2, 1000, 40959, 16777215):
            rec = O.draw(pairs, position, 1, seed=(seed & 0xFFFFFFFF, seed >> 32), top_k=40, temperature=0.8)
            assert rec[2] == _ref_uniform(seed, position + 1).view(np.uint32)
    for n in (2, 17, 512):
        rec = O.draw(pairs, 100, n, seed=(7, 0), top_k=40, temperature=0.8)
        assert rec[2] == _ref_uniform(7, 100 + n).view(np.uint32)


@needs_ref
def test_draw_equals_the_reference_f64_draw_given_its_uniform():
    """tests/gpu/draw_test.cpp:127-152 on the oracle: over five settings and
    200 positions each, the token drawn is the f64 reference's choice for the
    same uniform, except where the reference says the decision lies within
    f32 rounding (margin < 1e-5); those are at most 1% of the draws."""
    logits, tokens = _candidates(2)
    pairs = _pairs(logits, tokens)
    compared = near = 0
    for s in DRAW_SETTINGS:
        for position in range(200):
            rec = O.draw(pairs, position, 1, seed=(42, 0), temperature=s[0], top_k=s[1], top_p=s[2], min_p=s[3])
            assert rec[1] == 0
            chosen, margin = _ref_draw(logits, tokens, s, float(rec[2:3].view(np.float32)[0]))
            if margin < 1e-5:
                near += 1
                continue
            compared += 1
            assert rec[0] == tokens[chosen], (s, position)
    assert near * 100 <= compared


def test_draw_settings_at_their_edges():
    """tests/gpu/draw_test.cpp:154-175 on the oracle."""
    logits, tokens = _candidates(3)
    pairs = _pairs(logits, tokens)
    for position in range(20):
        for s in ((0.0, 40, 0.95, 0.05), (1.0, 1, 1.0, 0.0), (1.0, 64, 0.01, 0.0), (1.0, 64, 1.0, 0.99)):
            rec = O.draw(pairs, position, 1, seed=(9, 0), temperature=s[0], top_k=s[1], top_p=s[2], min_p=s[3])
            assert rec[0] == tokens[0]
    for position in range(50):
        rec = O.draw(pairs, position, 1, seed=(9, 0), temperature=100.0, top_k=2)
        assert rec[0] in (tokens[0], tokens[1])


def test_non_finite_top_candidate_fails_the_draw():
    """tests/gpu/draw_test.cpp:177-190 on the oracle: failed = 1, token 0."""
    for bad in (np.float32("nan"), np.float32("inf")):
        logits, tokens = _candidates(4)
        logits[0] = bad
        rec = O.draw(_pairs(logits, tokens), 0, 1, seed=(1, 0), temperature=0.8, top_k=40, top_p=0.95, min_p=0.05)
        assert rec[1] == 1 and rec[0] == 0
