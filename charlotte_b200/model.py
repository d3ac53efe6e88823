"""Decoder models on the C ABI: architecture presets with the shapes the
benchmark configurations name (Qwen3-0.6B, Llama-3.2-1B, Gemma-3-1B), seeded
random-init weights in GGUF blocks (synth.py), and a Decoder that uploads them
through cb_decoder_create and steps them (cb_decoder_step, cb_decoder_generate).
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass, field

import numpy as np

from . import synth
from . import lib as _lib, check as _check, CharlotteError  # noqa: F401

Q4_0, Q8_0, Q6_K = synth.Q4_0, synth.Q8_0, synth.Q6_K
SILU, GELU_TANH = 0, 1


@dataclass
class Arch:
    name: str
    layers: int
    hidden: int
    query_heads: int
    kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    context: int
    epsilon: float = 1e-6
    rope_base: float = 1e6
    window_rope_base: float = 1e4
    halves: bool = True
    qk_norm: bool = True
    post_norms: bool = False
    activation: int = SILU
    embed_scale: float = 1.0
    attention_scale: float = 0.0        # 0: 1/sqrt(head_dim)
    window: int = 0                     # sliding window (0: none)
    window_pattern: int = 0             # every n-th layer (n-1 mod n) is global
    llama3_factors: bool = False
    matmul_format: int = Q4_0
    down_format: int = 0                # the down projections' format (0: matmul_format)
    embed_format: int = Q6_K
    output_format: int = 0              # 0: tied to the embedding

    def layer_window(self, l: int) -> int:
        if self.window and self.window_pattern and l % self.window_pattern != self.window_pattern - 1:
            return self.window
        return self.context

    def layer_rope_base(self, l: int) -> float:
        return self.window_rope_base if self.layer_window(l) < self.context else self.rope_base


def qwen3_0_6b(context=4096):
    """28 layers, hidden 1024, GQA 16/8 x 128, QK-norm,
    RoPE 1e6, SwiGLU 3072, tied vocab 151936 (Q6_K), Q4_0 matmuls."""
    return Arch("qwen3-0.6b", 28, 1024, 16, 8, 128, 3072, 151936, context, 1e-6, 1e6)


def llama_3_2_1b(context=4096):
    """16 layers, hidden 2048, 32/8 x 64, SwiGLU 8192,
    vocab 128256, RoPE 5e5 with llama3 factors; Q4_0 with a Q6_K output layer."""
    return Arch("llama-3.2-1b", 16, 2048, 32, 8, 64, 8192, 128256, context, 1e-5, 5e5, halves=False,
                qk_norm=False, llama3_factors=True, embed_format=Q4_0, output_format=Q6_K)


def gemma_3_1b(context=2048):
    """26 layers, hidden 1152, 4/1 x 256, window 512 on 5
    of 6 layers, GeGLU-tanh 6912, pre/post norms, sqrt(H) embedding scale,
    vocab 262144 tied. The tied table is Q8_0: Q6_K super-blocks of 256 cannot
    tile rows of 1152."""
    return Arch("gemma-3-1b", 26, 1152, 4, 1, 256, 6912, 262144, context, 1e-6, 1e6, 1e4, post_norms=True,
                activation=GELU_TANH, embed_scale=float(np.sqrt(np.float32(1152))), window=512, window_pattern=6,
                embed_format=Q8_0)


def tiny(kind="qwen3", context=256):
    """Small models of each family for parity tests."""
    if kind == "qwen3":
        return Arch("tiny-qwen3", 2, 256, 4, 2, 64, 512, 1000, context)
    if kind == "llama":
        return Arch("tiny-llama", 2, 256, 4, 2, 64, 512, 1000, context, 1e-5, 5e5, halves=False, qk_norm=False,
                    llama3_factors=True, embed_format=Q4_0, output_format=Q6_K)
    if kind == "gemma3":
        return Arch("tiny-gemma3", 3, 256, 4, 1, 256, 512, 1000, context, 1e-6, 1e6, 1e4, post_norms=True,
                    activation=GELU_TANH, embed_scale=16.0, window=16, window_pattern=3, embed_format=Q8_0)
    raise ValueError(kind)


def llama3_factors(head_dim: int, base: float, factor=32.0, low=1.0, high=4.0, original=8192.0) -> np.ndarray:
    """rope_freqs for llama3 frequency scaling (the published rule; the
    reference only reads the tensor, src/core/arch/describe.cpp:257-261)."""
    out = np.empty(head_dim // 2, np.float32)
    for k in range(head_dim // 2):
        wavelen = 2 * math.pi / base ** (-2.0 * k / head_dim)
        if wavelen < original / high:
            out[k] = 1.0
        elif wavelen > original / low:
            out[k] = factor
        else:
            smooth = (original / wavelen - low) / (high - low)
            out[k] = 1.0 / ((1 - smooth) / factor + smooth)
    return out


@dataclass
class Weight:
    format: int
    rows: int
    cols: int
    stored: np.ndarray

    @property
    def blocks(self) -> int:
        return self.rows * self.cols // synth.BLOCK_WEIGHTS[self.format]


@dataclass
class Layer:
    attn_norm: np.ndarray
    q: Weight
    k: Weight
    v: Weight
    o: Weight
    q_norm: np.ndarray | None
    k_norm: np.ndarray | None
    post_attn_norm: np.ndarray | None
    ffn_norm: np.ndarray
    gate: Weight
    up: Weight
    down: Weight
    post_ffn_norm: np.ndarray | None
    window: int
    rope_base: float


@dataclass
class Model:
    arch: Arch
    token_embd: Weight
    output_norm: np.ndarray
    output: Weight | None
    layers: list = field(default_factory=list)
    factors: np.ndarray | None = None


def _gain(rng, n):
    return (1.0 + 0.05 * rng.standard_normal(n)).astype(np.float32)


def synthesize(arch: Arch, seed: int = 0) -> Model:
    """Seeded random-init weights of `arch`: matmuls in arch.matmul_format
    (Q4_0: d = |N(0, 0.02)|/8, uniform codes), the embedding and head in their
    formats, f32 norm gains near 1."""
    rng = np.random.default_rng(seed)
    H, d, F = arch.hidden, arch.head_dim, arch.ffn

    def w(fmt, rows, cols):
        return Weight(fmt, rows, cols, synth.blocks(rng, fmt, rows, cols))

    embd = w(arch.embed_format, arch.vocab, H)
    output = w(arch.output_format, arch.vocab, H) if arch.output_format else None
    layers = []
    for l in range(arch.layers):
        f = arch.matmul_format
        layers.append(Layer(
            _gain(rng, H), w(f, arch.query_heads * d, H), w(f, arch.kv_heads * d, H), w(f, arch.kv_heads * d, H),
            w(f, H, arch.query_heads * d),
            _gain(rng, d) if arch.qk_norm else None, _gain(rng, d) if arch.qk_norm else None,
            _gain(rng, H) if arch.post_norms else None, _gain(rng, H),
            w(f, F, H), w(f, F, H), w(arch.down_format or f, H, F), _gain(rng, H) if arch.post_norms else None,
            arch.layer_window(l), arch.layer_rope_base(l)))
    factors = llama3_factors(d, arch.rope_base) if arch.llama3_factors else None
    return Model(arch, embd, _gain(rng, H), output, layers, factors)


# ---- the C ABI's structs -------------------------------------------------------

class CWeight(ctypes.Structure):
    _fields_ = [("format", ctypes.c_uint32), ("rows", ctypes.c_uint32), ("cols", ctypes.c_uint32),
                ("stored_host", ctypes.c_void_p)]


class CLayer(ctypes.Structure):
    _fields_ = [("attn_norm", ctypes.c_void_p), ("q", CWeight), ("k", CWeight), ("v", CWeight), ("o", CWeight),
                ("q_norm", ctypes.c_void_p), ("k_norm", ctypes.c_void_p), ("post_attn_norm", ctypes.c_void_p),
                ("ffn_norm", ctypes.c_void_p), ("gate", CWeight), ("up", CWeight), ("down", CWeight),
                ("post_ffn_norm", ctypes.c_void_p), ("window", ctypes.c_uint32), ("rope_base", ctypes.c_float)]


class CModel(ctypes.Structure):
    _fields_ = [("layers", ctypes.c_uint32), ("hidden", ctypes.c_uint32), ("query_heads", ctypes.c_uint32),
                ("kv_heads", ctypes.c_uint32), ("head_dim", ctypes.c_uint32), ("ffn", ctypes.c_uint32),
                ("vocab", ctypes.c_uint32), ("context", ctypes.c_uint32), ("epsilon", ctypes.c_float),
                ("attention_scale", ctypes.c_float), ("embed_scale", ctypes.c_float), ("halves", ctypes.c_uint32),
                ("activation", ctypes.c_uint32), ("rope_factors", ctypes.c_void_p), ("token_embd", CWeight),
                ("output_norm", ctypes.c_void_p), ("output", CWeight), ("layer", ctypes.POINTER(CLayer))]


class CSampling(ctypes.Structure):
    _fields_ = [("seed0", ctypes.c_uint32), ("seed1", ctypes.c_uint32), ("top_k", ctypes.c_uint32),
                ("temperature", ctypes.c_float), ("top_p", ctypes.c_float), ("min_p", ctypes.c_float)]


def _ptr(a):
    return None if a is None else a.ctypes.data


def _cweight(w: Weight | None) -> CWeight:
    if w is None:
        return CWeight(0, 0, 0, None)
    return CWeight(w.format, w.rows, w.cols, w.stored.ctypes.data)


def attention_scale(arch: Arch) -> float:
    return arch.attention_scale or float(np.float32(1.0) / np.sqrt(np.float32(arch.head_dim)))


def to_c(model: Model):
    """The cb_model for `model` (and the arrays it points into, to keep alive)."""
    a = model.arch
    layers = (CLayer * a.layers)()
    for i, L in enumerate(model.layers):
        layers[i] = CLayer(_ptr(L.attn_norm), _cweight(L.q), _cweight(L.k), _cweight(L.v), _cweight(L.o),
                           _ptr(L.q_norm), _ptr(L.k_norm), _ptr(L.post_attn_norm), _ptr(L.ffn_norm),
                           _cweight(L.gate), _cweight(L.up), _cweight(L.down), _ptr(L.post_ffn_norm), L.window,
                           L.rope_base)
    m = CModel(a.layers, a.hidden, a.query_heads, a.kv_heads, a.head_dim, a.ffn, a.vocab, a.context, a.epsilon,
               attention_scale(a), a.embed_scale, int(a.halves), a.activation, _ptr(model.factors),
               _cweight(model.token_embd), _ptr(model.output_norm), _cweight(model.output), layers)
    return m, layers


class Decoder:
    """A model uploaded through the C ABI; steps run on the GPU."""

    def __init__(self, model: Model, max_step_tokens: int = 512, tensor_prefill: bool = False):
        L = _lib()
        L.cb_decoder_create.restype = ctypes.c_int
        L.cb_decoder_create.argtypes = [ctypes.POINTER(CModel), ctypes.c_uint32, ctypes.c_uint32,
                                        ctypes.POINTER(ctypes.c_void_p)]
        L.cb_decoder_destroy.argtypes = [ctypes.c_void_p]
        L.cb_decoder_step.restype = ctypes.c_int
        L.cb_decoder_step.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32,
                                      ctypes.c_uint32, ctypes.POINTER(CSampling), ctypes.c_void_p]
        L.cb_decoder_generate.restype = ctypes.c_int
        L.cb_decoder_generate.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.POINTER(CSampling),
                                          ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_float)]
        L.cb_decoder_logits.restype = ctypes.c_int
        L.cb_decoder_logits.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        self.lib = L
        self.model = model
        self.max_step_tokens = max_step_tokens
        cm, self._layers = to_c(model)
        self._cm = cm
        h = ctypes.c_void_p()
        flags = 1 if tensor_prefill else 0   # CB_DECODER_TENSOR_PREFILL
        _check(L.cb_decoder_create(ctypes.byref(cm), max_step_tokens, flags, ctypes.byref(h)))
        self.handle = h

    def close(self):
        if getattr(self, "handle", None):
            self.lib.cb_decoder_destroy(self.handle)
            self.handle = None

    def __del__(self):
        self.close()

    @staticmethod
    def sampling(temperature=0.0, top_k=1, top_p=1.0, min_p=0.0, seed=(0, 0)) -> CSampling:
        return CSampling(seed[0], seed[1], top_k, temperature, top_p, min_p)

    def step(self, ids, position: int, logits: bool = True, sampling: CSampling | None = None) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.uint32)
        rec = np.zeros(4, np.uint32)
        s = sampling or self.sampling()
        _check(self.lib.cb_decoder_step(self.handle, ids.ctypes.data, ids.size, position, int(logits),
                                        ctypes.byref(s), rec.ctypes.data))
        return rec

    def prefill(self, ids, position: int = 0, sampling: CSampling | None = None) -> np.ndarray:
        """Steps the prompt in blocks of max_step_tokens; the last step draws."""
        ids = np.ascontiguousarray(ids, np.uint32)
        rec = None
        for at in range(0, ids.size, self.max_step_tokens):
            part = ids[at: at + self.max_step_tokens]
            rec = self.step(part, position + at, logits=at + part.size >= ids.size, sampling=sampling)
        return rec

    def generate(self, steps: int, sampling: CSampling | None = None, timed: bool = False):
        """Fed greedy (or sampled) decode steps as one replayed CUDA graph.
        Returns (tokens, failed) or, when timed, (tokens, failed, device_ms)."""
        toks = np.zeros(steps, np.uint32)
        failed = np.zeros(steps, np.uint32)
        s = sampling or self.sampling()
        ms = ctypes.c_float(0.0)
        _check(self.lib.cb_decoder_generate(self.handle, steps, ctypes.byref(s), toks.ctypes.data,
                                            failed.ctypes.data, ctypes.byref(ms) if timed else None))
        return (toks, failed, ms.value) if timed else (toks, failed)

    def logits(self) -> np.ndarray:
        out = np.empty(self.model.arch.vocab, np.float32)
        _check(self.lib.cb_decoder_logits(self.handle, out.ctypes.data))
        return out


class BatchDecoder(Decoder):
    """`sequences` independent sequences in one decoder (cb_decoder_create_batch):
    prompts go in per sequence, then every sequence steps together, one token
    each at a common position — the products read the weights once for all
    rows. Each row's bits are those of its sequence decoded alone."""

    def __init__(self, model: Model, sequences: int, max_step_tokens: int = 512, tensor_prefill: bool = False):
        L = _lib()
        L.cb_decoder_create_batch.restype = ctypes.c_int
        L.cb_decoder_create_batch.argtypes = [ctypes.POINTER(CModel), ctypes.c_uint32, ctypes.c_uint32,
                                              ctypes.c_uint32, ctypes.POINTER(ctypes.c_void_p)]
        L.cb_decoder_step_sequence.restype = ctypes.c_int
        L.cb_decoder_step_sequence.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_uint32,
                                               ctypes.c_uint32, ctypes.c_uint32, ctypes.POINTER(CSampling),
                                               ctypes.c_void_p]
        L.cb_decoder_step_batch.restype = ctypes.c_int
        L.cb_decoder_step_batch.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32,
                                            ctypes.POINTER(CSampling), ctypes.c_void_p]
        L.cb_decoder_logits_row.restype = ctypes.c_int
        L.cb_decoder_logits_row.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p]
        # the one-sequence bindings (destroy, generate, logits) come from Decoder
        L.cb_decoder_create.restype = ctypes.c_int
        L.cb_decoder_destroy.argtypes = [ctypes.c_void_p]
        L.cb_decoder_generate.restype = ctypes.c_int
        L.cb_decoder_generate.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.POINTER(CSampling),
                                          ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_float)]
        self.lib = L
        self.model = model
        self.sequences = sequences
        self.max_step_tokens = max_step_tokens
        cm, self._layers = to_c(model)
        self._cm = cm
        h = ctypes.c_void_p()
        flags = 1 if tensor_prefill else 0
        _check(L.cb_decoder_create_batch(ctypes.byref(cm), max_step_tokens, sequences, flags, ctypes.byref(h)))
        self.handle = h

    def step_sequence(self, seq: int, ids, position: int, logits: bool = True,
                      sampling: CSampling | None = None) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.uint32)
        rec = np.zeros(4, np.uint32)
        s = sampling or self.sampling()
        _check(self.lib.cb_decoder_step_sequence(self.handle, seq, ids.ctypes.data, ids.size, position, int(logits),
                                                 ctypes.byref(s), rec.ctypes.data))
        return rec

    def prefill_sequence(self, seq: int, ids, position: int = 0, sampling: CSampling | None = None) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.uint32)
        rec = None
        for at in range(0, ids.size, self.max_step_tokens):
            part = ids[at: at + self.max_step_tokens]
            rec = self.step_sequence(seq, part, position + at, logits=at + part.size >= ids.size, sampling=sampling)
        return rec

    def step_batch(self, ids, position: int, sampling: CSampling | None = None) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.uint32)
        assert ids.size == self.sequences
        recs = np.zeros((self.sequences, 4), np.uint32)
        s = sampling or self.sampling()
        _check(self.lib.cb_decoder_step_batch(self.handle, ids.ctypes.data, position, ctypes.byref(s),
                                              recs.ctypes.data))
        return recs

    def generate(self, steps: int, sampling: CSampling | None = None, timed: bool = False):
        """Fed batched steps as one replayed CUDA graph: tokens [steps, sequences]."""
        toks = np.zeros((steps, self.sequences), np.uint32)
        failed = np.zeros((steps, self.sequences), np.uint32)
        s = sampling or self.sampling()
        ms = ctypes.c_float(0.0)
        _check(self.lib.cb_decoder_generate(self.handle, steps, ctypes.byref(s), toks.ctypes.data,
                                            failed.ctypes.data, ctypes.byref(ms) if timed else None))
        return (toks, failed, ms.value) if timed else (toks, failed)

    def logits_row(self, row: int) -> np.ndarray:
        out = np.empty(self.model.arch.vocab, np.float32)
        _check(self.lib.cb_decoder_logits_row(self.handle, row, out.ctypes.data))
        return out
