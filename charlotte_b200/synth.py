"""Seeded synthetic GGUF weights with the shapes and value distributions the
benchmark configurations name (random-init weights; there are no real model
files on these machines).

Blocks are generated in the stored (file) order of ggml's block structs —
Q4_0 {d: f16, qs[16]}, Q4_1 {d: f16, m: f16, qs[16]}, Q8_0 {d: f16,
qs[32]}, Q6_K {ql[128], qh[64], scales[16]: i8, d: f16}, BF16 values — and
turned into the device layout by `to_piece`.
"""
from __future__ import annotations

import numpy as np

F32, F16, Q4_0, Q4_1, Q8_0, Q6_K, BF16 = 0, 1, 2, 3, 8, 14, 30
BLOCK_BYTES = {F32: 4, F16: 2, Q4_0: 18, Q4_1: 20, Q8_0: 34, Q6_K: 210, BF16: 2}
BLOCK_WEIGHTS = {F32: 1, F16: 1, Q4_0: 32, Q4_1: 32, Q8_0: 32, Q6_K: 256, BF16: 1}


def _fp16_bits(values: np.ndarray) -> np.ndarray:
    return np.asarray(values, np.float32).astype(np.float16).view(np.uint16)


def q4_0_blocks(rng: np.random.Generator, n_blocks: int, sigma: float = 0.02) -> np.ndarray:
    """d = |N(0, sigma)|/8 as f16, 16 bytes of uniform codes (value (q-8)*d)."""
    out = np.empty((n_blocks, 18), np.uint8)
    d = _fp16_bits(np.abs(rng.normal(0.0, sigma, n_blocks)) / 8.0)
    out[:, 0:2] = d.view(np.uint8).reshape(n_blocks, 2)
    out[:, 2:] = rng.integers(0, 256, (n_blocks, 16), dtype=np.uint8)
    return out.reshape(-1)


def q4_1_blocks(rng: np.random.Generator, n_blocks: int, sigma: float = 0.02) -> np.ndarray:
    """d = |N(0, sigma)|/8 and m = -7.5*d*(1 + N(0, 0.05)) as f16, 16 bytes of
    uniform codes (value q*d + m)."""
    out = np.empty((n_blocks, 20), np.uint8)
    d = np.abs(rng.normal(0.0, sigma, n_blocks)) / 8.0
    m = -7.5 * d * (1.0 + rng.normal(0.0, 0.05, n_blocks))
    out[:, 0:2] = _fp16_bits(d).view(np.uint8).reshape(n_blocks, 2)
    out[:, 2:4] = _fp16_bits(m).view(np.uint8).reshape(n_blocks, 2)
    out[:, 4:] = rng.integers(0, 256, (n_blocks, 16), dtype=np.uint8)
    return out.reshape(-1)


def bf16_values(rng: np.random.Generator, n: int, sigma: float = 0.02) -> np.ndarray:
    """N(0, sigma) rounded to bfloat16 (nearest, ties to even), 2 bytes each."""
    bits = rng.normal(0.0, sigma, n).astype(np.float32).view(np.uint32)
    rounded = (bits + 0x7FFF + ((bits >> 16) & 1)) >> 16
    return rounded.astype(np.uint16).view(np.uint8)


def q8_0_blocks(rng: np.random.Generator, n_blocks: int, sigma: float = 0.02) -> np.ndarray:
    """d = |N(0, sigma)|/127 as f16, 32 uniform int8 codes."""
    out = np.empty((n_blocks, 34), np.uint8)
    d = _fp16_bits(np.abs(rng.normal(0.0, sigma, n_blocks)) / 127.0)
    out[:, 0:2] = d.view(np.uint8).reshape(n_blocks, 2)
    out[:, 2:] = rng.integers(0, 256, (n_blocks, 32), dtype=np.uint8)
    return out.reshape(-1)


def q6_k_blocks(rng: np.random.Generator, n_blocks: int, sigma: float = 0.02) -> np.ndarray:
    """Random ql (128 B), qh (64 B), int8 scales (16) and f16 d = |N(0,sigma)|/2048."""
    out = np.empty((n_blocks, 210), np.uint8)
    out[:, :192] = rng.integers(0, 256, (n_blocks, 192), dtype=np.uint8)
    out[:, 192:208] = rng.integers(-127, 128, (n_blocks, 16)).astype(np.int8).view(np.uint8)
    d = _fp16_bits(np.abs(rng.normal(0.0, sigma, n_blocks)) / 2048.0)
    out[:, 208:210] = d.view(np.uint8).reshape(n_blocks, 2)
    return out.reshape(-1)


def random_bytes_blocks(rng: np.random.Generator, fmt: int, n_blocks: int) -> np.ndarray:
    """Uniformly random block bytes whose f16 scales are finite: every code,
    every scale class (subnormal, zero, negative) — the unpack edge cases."""
    bb = BLOCK_BYTES[fmt]
    out = rng.integers(0, 256, (n_blocks, bb), dtype=np.uint8)
    if fmt == BF16:
        # clear the exponent's lowest bit where all eight are ones
        exp_all_ones = ((out[:, 1] & 0x7F) == 0x7F) & ((out[:, 0] & 0x80) != 0)
        out[exp_all_ones, 0] &= 0x7F
        return out.reshape(-1)
    for at in ((208,) if fmt == Q6_K else ((0, 2) if fmt == Q4_1 else (0,))):
        # clear exponent bit 14 of an f16 field when the exponent would be 31
        hi = out[:, at + 1]
        exp_all_ones = (hi & 0x7C) == 0x7C
        out[exp_all_ones, at + 1] = hi[exp_all_ones] & 0xFB
    return out.reshape(-1)


def blocks(rng: np.random.Generator, fmt: int, rows: int, cols: int) -> np.ndarray:
    n = rows * cols // BLOCK_WEIGHTS[fmt]
    if fmt == Q4_0:
        return q4_0_blocks(rng, n)
    if fmt == Q4_1:
        return q4_1_blocks(rng, n)
    if fmt == BF16:
        return bf16_values(rng, n)
    if fmt == Q8_0:
        return q8_0_blocks(rng, n)
    if fmt == Q6_K:
        return q6_k_blocks(rng, n)
    raise ValueError(f"format {fmt}")


def piece_bytes(fmt: int, n_blocks: int) -> int:
    return (n_blocks * BLOCK_BYTES[fmt] + 15) // 16 * 16


def to_piece(fmt: int, stored: np.ndarray) -> np.ndarray:
    """Stored blocks -> the device layout: each field a stream over every block
    (Q4_0/Q8_0 codes then scales; Q6_K repacked low nibbles, high pairs,
    scales, d), padded to 16 bytes."""
    bb = BLOCK_BYTES[fmt]
    st = np.ascontiguousarray(stored, np.uint8).reshape(-1, bb)
    n = st.shape[0]
    out = np.zeros(piece_bytes(fmt, n), np.uint8)
    if fmt in (Q4_0, Q8_0):
        cb = bb - 2
        out[: cb * n] = st[:, 2:].reshape(-1)
        out[cb * n: cb * n + 2 * n] = st[:, :2].reshape(-1)
        return out
    if fmt == Q6_K:
        ql = st[:, :128].astype(np.uint32)
        qh = st[:, 128:192].astype(np.uint32)
        lo = np.zeros((n, 8, 16), np.uint32)
        hi = np.zeros((n, 8, 8), np.uint32)
        l = np.arange(32)
        for k in range(8):
            h, r = divmod(k, 4)
            nib = (ql[:, 64 * h + 32 * (r % 2) + l] >> (4 * (r // 2))) & 0xF
            pair = (qh[:, 32 * h + l] >> (2 * r)) & 3
            for li in range(32):
                lo[:, k, li % 16] |= nib[:, li] << (4 * (li // 16))
                hi[:, k, li % 8] |= pair[:, li] << (2 * (li // 8))
        out[: 128 * n] = lo.astype(np.uint8).reshape(-1)
        out[128 * n: 192 * n] = hi.astype(np.uint8).reshape(-1)
        out[192 * n: 208 * n] = st[:, 192:208].reshape(-1)
        out[208 * n: 210 * n] = st[:, 208:210].reshape(-1)
        return out
    if fmt == Q4_1:   # codes, then each block's (d, m) word
        out[: 16 * n] = st[:, 4:].reshape(-1)
        out[16 * n: 20 * n] = st[:, :4].reshape(-1)
        return out
    if fmt in (F32, F16, BF16):
        out[: bb * n] = st.reshape(-1)
        return out
    raise ValueError(f"format {fmt}")


def activations(rng: np.random.Generator, tokens: int, k: int) -> np.ndarray:
    return rng.standard_normal((tokens, k)).astype(np.float32)
