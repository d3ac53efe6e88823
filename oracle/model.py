"""The oracle's whole decoder pass (oracle.c or_forward) over the same
synthetic model the CUDA decoder runs — TEST INFRASTRUCTURE ONLY."""
from __future__ import annotations

import ctypes

import numpy as np

from . import lib, to_piece, rope_turns, DrawSettings


class OWeight(ctypes.Structure):
    _fields_ = [("type", ctypes.c_int), ("piece", ctypes.c_void_p), ("blocks", ctypes.c_uint32),
                ("rows", ctypes.c_uint32), ("cols", ctypes.c_uint32)]


class OLayer(ctypes.Structure):
    _fields_ = [("attn_norm", ctypes.c_void_p), ("q", OWeight), ("k", OWeight), ("v", OWeight), ("o", OWeight),
                ("q_norm", ctypes.c_void_p), ("k_norm", ctypes.c_void_p), ("post_attn_norm", ctypes.c_void_p),
                ("ffn_norm", ctypes.c_void_p), ("gate", OWeight), ("up", OWeight), ("down", OWeight),
                ("post_ffn_norm", ctypes.c_void_p), ("window", ctypes.c_uint32), ("slots", ctypes.c_uint32),
                ("turns", ctypes.c_void_p)]


class OModel(ctypes.Structure):
    _fields_ = [("layers", ctypes.c_uint32), ("hidden", ctypes.c_uint32), ("query_heads", ctypes.c_uint32),
                ("kv_heads", ctypes.c_uint32), ("head_dim", ctypes.c_uint32), ("ffn", ctypes.c_uint32),
                ("vocab", ctypes.c_uint32), ("epsilon", ctypes.c_float), ("attention_scale", ctypes.c_float),
                ("embed_scale", ctypes.c_float), ("halves", ctypes.c_int), ("activation", ctypes.c_int),
                ("factors", ctypes.c_void_p), ("token_embd", OWeight), ("output_norm", ctypes.c_void_p),
                ("output", OWeight), ("layer", ctypes.POINTER(OLayer))]


def _p(a):
    return None if a is None else a.ctypes.data


class OracleDecoder:
    """Steps a charlotte_b200.model.Model on the CPU in the reference's order."""

    def __init__(self, model, threads: int = 0):
        import os
        from charlotte_b200.model import attention_scale
        self.model = model
        self.threads = threads or os.cpu_count() or 1
        a = model.arch
        self._keep = []

        def w(x):
            if x is None:
                return OWeight(0, None, 0, 0, 0)
            piece = to_piece(x.format, x.stored)
            self._keep.append(piece)
            return OWeight(x.format, piece.ctypes.data, x.blocks, x.rows, x.cols)

        layers = (OLayer * a.layers)()
        for i, L in enumerate(model.layers):
            turns = rope_turns(L.rope_base, a.head_dim)
            self._keep.append(turns)
            layers[i] = OLayer(_p(L.attn_norm), w(L.q), w(L.k), w(L.v), w(L.o), _p(L.q_norm), _p(L.k_norm),
                               _p(L.post_attn_norm), _p(L.ffn_norm), w(L.gate), w(L.up), w(L.down),
                               _p(L.post_ffn_norm), L.window, a.context, turns.ctypes.data)
        embd = w(model.token_embd)
        out = w(model.output) if model.output is not None else embd
        self._layers = layers
        self._m = OModel(a.layers, a.hidden, a.query_heads, a.kv_heads, a.head_dim, a.ffn, a.vocab, a.epsilon,
                         attention_scale(a), a.embed_scale, int(a.halves), a.activation, _p(model.factors), embd,
                         _p(model.output_norm), out, layers)
        L = lib()
        L.or_state_create.restype = ctypes.c_void_p
        L.or_state_create.argtypes = [ctypes.POINTER(OModel)]
        L.or_state_destroy.argtypes = [ctypes.c_void_p]
        L.or_forward.restype = ctypes.c_int
        L.or_forward.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_int,
                                 ctypes.POINTER(DrawSettings), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
        self.lib = L
        self.state = L.or_state_create(ctypes.byref(self._m))

    def close(self):
        if self.state:
            self.lib.or_state_destroy(self.state)
            self.state = None

    def __del__(self):
        self.close()

    def step(self, ids, position, logits=True, temperature=0.0, top_k=1, top_p=1.0, min_p=0.0, seed=(0, 0)):
        """Returns (record, logits or None)."""
        import math
        ids = np.ascontiguousarray(ids, np.uint32)
        rec = np.zeros(4, np.uint32)
        lg = np.zeros(self.model.arch.vocab, np.float32) if logits else None
        s = DrawSettings(position, ids.size, seed[0], seed[1], top_k, temperature, top_p, min_p,
                         math.log(min_p) if min_p > 0 else 0.0)
        rc = self.lib.or_forward(self.state, ids.ctypes.data, ids.size, position, int(logits), ctypes.byref(s),
                                 lg.ctypes.data if lg is not None else None, rec.ctypes.data, self.threads)
        assert rc == 0
        return rec, lg
