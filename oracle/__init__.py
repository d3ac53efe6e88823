"""ctypes bindings for the CPU oracle (oracle.c) and for oracle/_ref, the
reference's own CPU code compiled from its sources — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this package; the product (charlotte_b200) never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libcharlotte_ref.so")

F32, F16, Q4_0, Q4_1, Q8_0, Q6_K, BF16 = 0, 1, 2, 3, 8, 14, 30
SILU, GELU_TANH, SIGMOID = 0, 1, 2
BLOCK_BYTES = {F32: 4, F16: 2, Q4_0: 18, Q4_1: 20, Q8_0: 34, Q6_K: 210, BF16: 2}
BLOCK_WEIGHTS = {F32: 1, F16: 1, Q4_0: 32, Q4_1: 32, Q8_0: 32, Q6_K: 256, BF16: 1}

_lib = None
_ref = None

c_u8p = ctypes.POINTER(ctypes.c_uint8)
c_f32p = ctypes.POINTER(ctypes.c_float)
c_u16p = ctypes.POINTER(ctypes.c_uint16)
c_u32p = ctypes.POINTER(ctypes.c_uint32)


def reference_root() -> str | None:
    """The reference project's root: $CHARLOTTE_REFERENCE, else the
    `reference_path` BASELINE.json records; None where neither names an
    existing directory (a GPU box, which carries the prebuilt oracle/_ref)."""
    root = os.environ.get("CHARLOTTE_REFERENCE")
    if not root:
        import json
        try:
            with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as fh:
                root = json.load(fh).get("reference_path")
        except (OSError, ValueError):
            root = None
    return root if root and os.path.isdir(root) else None


def build() -> None:
    """Compile liboracle.so (and oracle/_ref when the reference is present)."""
    subprocess.run(["make", "-s", "-C", HERE, "liboracle.so"], check=True)
    root = reference_root()
    if root:
        subprocess.run(["make", "-s", "-C", HERE, "ref", "REF=" + root], check=True)


def ptr(a: np.ndarray, ctype):
    return a.ctypes.data_as(ctypes.POINTER(ctype))


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.or_fp16_to_fp32.restype = ctypes.c_float
        L.or_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        L.or_fp32_to_fp16_sat.restype = ctypes.c_uint16
        L.or_fp32_to_fp16_sat.argtypes = [ctypes.c_float]
        for name in ("or_exp_nonpositive", "or_exp2"):
            getattr(L, name).restype = ctypes.c_float
            getattr(L, name).argtypes = [ctypes.c_float]
        L.or_activate.restype = ctypes.c_float
        L.or_activate.argtypes = [ctypes.c_int, ctypes.c_float]
        L.or_sincos.argtypes = [ctypes.c_float, c_f32p, c_f32p]
        L.or_dequant_stored.argtypes = [ctypes.c_int, c_u8p, ctypes.c_size_t, c_f32p]
        L.or_piece_bytes.restype = ctypes.c_size_t
        L.or_piece_bytes.argtypes = [ctypes.c_int, ctypes.c_size_t]
        L.or_to_piece.argtypes = [ctypes.c_int, c_u8p, ctypes.c_size_t, c_u8p]
        L.or_unpack.argtypes = [ctypes.c_int, c_u8p, ctypes.c_uint32, ctypes.c_uint32, c_f32p]
        L.or_matmul.argtypes = [ctypes.c_int, c_u8p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                ctypes.c_uint32, c_f32p, ctypes.c_uint32, c_f32p, ctypes.c_uint32, ctypes.c_int]
        L.or_norm_row.argtypes = [c_f32p, c_f32p, c_f32p, c_f32p, ctypes.c_uint32, ctypes.c_float,
                                  ctypes.c_int, c_f32p]
        L.or_rope_turns.argtypes = [ctypes.c_double, ctypes.c_uint32, c_f32p]
        L.or_topk64.argtypes = [c_f32p, ctypes.c_uint32, c_u32p]
        L.or_philox4x32_10.argtypes = [c_u32p, c_u32p, c_u32p]
        L.or_attention_row.argtypes = [c_f32p, ctypes.c_uint32, c_u16p, c_u16p, ctypes.c_uint32,
                                       ctypes.c_uint32, ctypes.c_float, ctypes.c_uint32, ctypes.c_uint32,
                                       ctypes.c_uint32, c_f32p]
        _lib = L
    return _lib


def ref():
    """The reference's own CPU code (oracle/_ref), or None where it was not built."""
    global _ref
    if _ref is None and os.path.exists(REF_PATH):
        R = ctypes.CDLL(REF_PATH)
        for name in ("ref_dequant_q4_0", "ref_dequant_q8_0", "ref_dequant_q6_k", "ref_dequant_q4_1_fused",
                     "ref_dequant_q4_1_rounded"):
            getattr(R, name).restype = ctypes.c_int
            getattr(R, name).argtypes = [c_u8p, ctypes.c_size_t, c_f32p]
        R.ref_fp16_to_fp32.restype = ctypes.c_float
        R.ref_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        R.ref_fp32_to_fp16_saturating.restype = ctypes.c_uint16
        R.ref_fp32_to_fp16_saturating.argtypes = [ctypes.c_float]
        R.ref_repack_q6_k.argtypes = [c_u8p, ctypes.c_size_t, c_u8p, c_u8p, c_u8p, c_u8p]
        R.ref_philox.argtypes = [c_u32p, ctypes.c_uint32, ctypes.c_uint32, c_u32p]
        _ref = R
    return _ref


# ---- numpy helpers ----------------------------------------------------------

def dequant_stored(fmt: int, stored: np.ndarray) -> np.ndarray:
    stored = np.ascontiguousarray(stored, dtype=np.uint8)
    blocks = stored.size // BLOCK_BYTES[fmt]
    out = np.empty(blocks * BLOCK_WEIGHTS[fmt], np.float32)
    rc = lib().or_dequant_stored(fmt, ptr(stored, ctypes.c_uint8), blocks, ptr(out, ctypes.c_float))
    assert rc == 0
    return out


def to_piece(fmt: int, stored: np.ndarray) -> np.ndarray:
    stored = np.ascontiguousarray(stored, dtype=np.uint8)
    blocks = stored.size // BLOCK_BYTES[fmt]
    out = np.zeros(lib().or_piece_bytes(fmt, blocks), np.uint8)
    assert lib().or_to_piece(fmt, ptr(stored, ctypes.c_uint8), blocks, ptr(out, ctypes.c_uint8)) == 0
    return out


def unpack(fmt: int, piece: np.ndarray, blocks: int, group: int) -> np.ndarray:
    out = np.empty(32, np.float32)
    assert lib().or_unpack(fmt, ptr(piece, ctypes.c_uint8), blocks, group, ptr(out, ctypes.c_float)) == 0
    return out


def matmul(fmt: int, piece: np.ndarray, blocks: int, rows: int, K: int, x: np.ndarray,
           threads: int = 0) -> np.ndarray:
    """y[t, o] in the reference's order; x is [tokens, K] float32."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, K)
    tokens = x.shape[0]
    y = np.empty((tokens, rows), np.float32)
    threads = threads or os.cpu_count() or 1
    rc = lib().or_matmul(fmt, ptr(piece, ctypes.c_uint8), blocks, 0, rows, K, ptr(x, ctypes.c_float), tokens,
                         ptr(y, ctypes.c_float), rows, threads)
    assert rc == 0
    return y


def norm_row(hidden: np.ndarray, output, gain: np.ndarray, post_gain, epsilon: float, add: bool):
    """Returns (new hidden, normed) for one row."""
    h = np.array(hidden, np.float32, copy=True)
    width = h.size
    normed = np.empty(width, np.float32)
    out = np.ascontiguousarray(output if output is not None else np.zeros(width), np.float32)
    g = np.ascontiguousarray(gain, np.float32)
    pg = np.ascontiguousarray(post_gain, np.float32) if post_gain is not None else None
    lib().or_norm_row(ptr(h, ctypes.c_float), ptr(out, ctypes.c_float), ptr(g, ctypes.c_float),
                      ptr(pg, ctypes.c_float) if pg is not None else None, width, epsilon, int(add),
                      ptr(normed, ctypes.c_float))
    return h, normed


def norm_row_ex(hidden, output, gain, *, epsilon, add=True, post_gain=None, post_scale=1.0, scale=None,
                normalize=True):
    """norm.wgsl with the encoder's variants (or_norm_row_ex), one row:
    returns (new hidden, normed or None). gain None: no gain."""
    h = np.array(hidden, np.float32, copy=True)
    width = h.size
    normed = np.empty(width, np.float32)
    out = np.ascontiguousarray(output if output is not None else np.zeros(width), np.float32)
    keep = [np.ascontiguousarray(a, np.float32) if a is not None else None for a in (gain, post_gain, scale)]
    L = lib()
    L.or_norm_row_ex.argtypes = [c_f32p, c_f32p, c_f32p, c_f32p, ctypes.c_float, c_f32p, ctypes.c_uint32,
                                 ctypes.c_float, ctypes.c_int, ctypes.c_int, c_f32p]
    L.or_norm_row_ex(ptr(h, ctypes.c_float), ptr(out, ctypes.c_float),
                     *[ptr(a, ctypes.c_float) if a is not None else None for a in keep[:2]], post_scale,
                     ptr(keep[2], ctypes.c_float) if keep[2] is not None else None, width, epsilon, int(add),
                     int(normalize), ptr(normed, ctypes.c_float))
    return h, (normed if normalize else None)


def rope_encode_token(q, k, v, p, *, head_dim, query_heads, kv_heads, halves, epsilon, turns, factors=None,
                      query_gain=None, key_gain=None, value_norm=False):
    """rope_encode.wgsl for one token, q, k and v (f32 [heads*d]) in place."""
    keep = [np.ascontiguousarray(a, np.float32) if a is not None else None
            for a in (turns, factors, query_gain, key_gain)]
    s = RopeShape(head_dim, query_heads, kv_heads, int(halves), int(query_gain is not None), 1, epsilon,
                  *[ptr(a, ctypes.c_float) if a is not None else None for a in keep])
    L = lib()
    L.or_rope_encode_token.argtypes = [ctypes.POINTER(RopeShape), ctypes.c_uint32, ctypes.c_int, c_f32p, c_f32p,
                                       c_f32p]
    L.or_rope_encode_token(ctypes.byref(s), p, int(value_norm), ptr(q, ctypes.c_float), ptr(k, ctypes.c_float),
                           ptr(v, ctypes.c_float))


def block_attention(q, k, v, *, tokens, head_dim, query_heads, kv_heads, half_window, scale_log2e):
    """block_attention.wgsl scores_of + weigh over a step: q [n][hq*d], k, v
    [n][hkv*d] -> out [n][hq*d]."""
    qq, kk, vv = (np.ascontiguousarray(a, np.float32) for a in (q, k, v))
    out = np.empty((tokens, query_heads * head_dim), np.float32)
    L = lib()
    L.or_block_attention.argtypes = [c_f32p, c_f32p, c_f32p] + [ctypes.c_uint32] * 5 + [ctypes.c_float, c_f32p]
    L.or_block_attention(ptr(qq, ctypes.c_float), ptr(kk, ctypes.c_float), ptr(vv, ctypes.c_float), tokens,
                         head_dim, query_heads, kv_heads, half_window, scale_log2e, ptr(out, ctypes.c_float))
    return out


def pool_mean(rows):
    """pool.wgsl mean over the rows of a [n][width] array."""
    r = np.ascontiguousarray(rows, np.float32)
    out = np.empty(r.shape[1], np.float32)
    L = lib()
    L.or_pool_mean.argtypes = [c_f32p, ctypes.c_uint32, ctypes.c_uint32, c_f32p]
    L.or_pool_mean(ptr(r, ctypes.c_float), r.shape[0], r.shape[1], ptr(out, ctypes.c_float))
    return out


def pool_unit(row):
    """pool.wgsl unit: the row over its Euclidean length."""
    r = np.ascontiguousarray(row, np.float32)
    out = np.empty(r.size, np.float32)
    L = lib()
    L.or_pool_unit.argtypes = [c_f32p, ctypes.c_uint32, c_f32p]
    L.or_pool_unit(ptr(r, ctypes.c_float), r.size, ptr(out, ctypes.c_float))
    return out


def rope_turns(base: float, head_dim: int) -> np.ndarray:
    t = np.empty(head_dim // 2, np.float32)
    lib().or_rope_turns(base, head_dim, ptr(t, ctypes.c_float))
    return t


def topk64(logits: np.ndarray) -> np.ndarray:
    logits = np.ascontiguousarray(logits, np.float32)
    out = np.empty(128, np.uint32)
    lib().or_topk64(ptr(logits, ctypes.c_float), logits.size, ptr(out, ctypes.c_uint32))
    return out


def philox(counter, key) -> np.ndarray:
    c = np.array(counter, np.uint32)
    k = np.array(key, np.uint32)
    out = np.empty(4, np.uint32)
    lib().or_philox4x32_10(ptr(c, ctypes.c_uint32), ptr(k, ctypes.c_uint32), ptr(out, ctypes.c_uint32))
    return out


def attention_row(q, p, key_cache, value_cache, slots, window, scale_log2e, head_dim, query_heads, kv_heads):
    q = np.ascontiguousarray(q, np.float32)
    out = np.empty(query_heads * head_dim, np.float32)
    lib().or_attention_row(ptr(q, ctypes.c_float), p, ptr(key_cache, ctypes.c_uint16),
                           ptr(value_cache, ctypes.c_uint16), slots, window, scale_log2e, head_dim,
                           query_heads, kv_heads, ptr(out, ctypes.c_float))
    return out


class RopeShape(ctypes.Structure):
    _fields_ = [("head_dim", ctypes.c_uint32), ("query_heads", ctypes.c_uint32), ("kv_heads", ctypes.c_uint32),
                ("halves", ctypes.c_int), ("qk_norm", ctypes.c_int), ("slots", ctypes.c_uint32),
                ("epsilon", ctypes.c_float), ("turns", c_f32p), ("factors", c_f32p),
                ("query_gain", c_f32p), ("key_gain", c_f32p)]


class DrawSettings(ctypes.Structure):
    _fields_ = [("position", ctypes.c_uint32), ("tokens", ctypes.c_uint32), ("seed0", ctypes.c_uint32),
                ("seed1", ctypes.c_uint32), ("top_k", ctypes.c_uint32), ("temperature", ctypes.c_float),
                ("top_p", ctypes.c_float), ("min_p", ctypes.c_float), ("log_min_p", ctypes.c_float)]


def rope_token(q, k, v, p, key_cache, value_cache, *, head_dim, query_heads, kv_heads, halves, slots, epsilon,
               turns, factors=None, query_gain=None, key_gain=None):
    """One token in place: q (f32 [Hq*d]) rotated; k, v packed into the caches."""
    keep = [np.ascontiguousarray(a, np.float32) if a is not None else None
            for a in (turns, factors, query_gain, key_gain)]
    s = RopeShape(head_dim, query_heads, kv_heads, int(halves), int(query_gain is not None), slots, epsilon,
                  *[ptr(a, ctypes.c_float) if a is not None else None for a in keep])
    L = lib()
    L.or_rope_token.argtypes = [ctypes.POINTER(RopeShape), ctypes.c_uint32, c_f32p, c_f32p, c_f32p, c_u16p, c_u16p]
    kk = np.ascontiguousarray(k, np.float32)
    vv = np.ascontiguousarray(v, np.float32)
    L.or_rope_token(ctypes.byref(s), p, ptr(q, ctypes.c_float), ptr(kk, ctypes.c_float), ptr(vv, ctypes.c_float),
                    ptr(key_cache, ctypes.c_uint16), ptr(value_cache, ctypes.c_uint16))


def draw(pairs128, position, tokens, seed=(0, 0), top_k=40, temperature=0.0, top_p=1.0, min_p=0.0):
    import math
    s = DrawSettings(position, tokens, seed[0], seed[1], top_k, temperature, top_p, min_p,
                     math.log(min_p) if min_p > 0 else 0.0)
    pairs = np.ascontiguousarray(pairs128, np.uint32)
    rec = np.zeros(4, np.uint32)
    L = lib()
    L.or_draw.argtypes = [c_u32p, ctypes.POINTER(DrawSettings), c_u32p]
    L.or_draw(ptr(pairs, ctypes.c_uint32), ctypes.byref(s), ptr(rec, ctypes.c_uint32))
    return rec
