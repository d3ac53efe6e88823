"""A synthetic EmbeddingGemma 2 text encoder — TEST INFRASTRUCTURE: seeded
random-init weights of the `gemma-embedding2` architecture, written as a
GGUF v3 file with the keys and tensors the reference's description reads
(src/core/arch/embedding_gemma2/embedding_gemma2.cpp:69-172,
src/core/arch/describe.cpp:133-290), and the oracle's pass over it in the
order src/core/graph/encoder.h:38-110 and encoder.cpp:198-376 lay out:

  embed (× √W) → per-layer inputs (one product, each P-wide slice normed
  with ε·W) → per layer: attention (norm adding the pending block, QKV,
  rope's encode form, block attention, output), gated feed-forward,
  per-layer block (add alone, gelu(W x) ⊙ the layer's per-layer input,
  projection; its post-norm and the layer's output scale pending) → the
  final norm over every row, the mean, the output projection of that one
  row, unit length."""
from __future__ import annotations

import math
import struct
from dataclasses import dataclass, field

import numpy as np

import oracle as O
from charlotte_b200 import synth
from gguf_writer import ALIGNMENT, T_F32, U32, F32, STRING, ARRAY, _kv, _string, _u32, _f32, _str, _strings

BOOL = 7
ARCH = "gemma-embedding2"
GELU_TANH = 1
Q4_0, Q8_0 = 2, 8


@dataclass
class EncoderArch:
    layers: int = 2
    hidden: int = 256          # W
    query_heads: int = 4
    kv_heads: int = 1
    head_dim: int = 256        # the sliding layers' heads
    global_head_dim: int = 512  # the global layers' (EmbeddingGemma 2's)
    ffn: int = 512
    vocab: int = 300
    per_layer: int = 64        # P
    embedding: int = 128       # E
    window: int = 64           # the sliding layers' (half of it either side)
    sliding: list = field(default_factory=lambda: [True, False])
    context: int = 512
    epsilon: float = 1e-6
    rope_base: float = 1_000_000.0
    swa_base: float = 10_000.0


@dataclass
class W:
    format: int
    rows: int
    cols: int
    stored: np.ndarray

    @property
    def blocks(self):
        return self.rows * self.cols // synth.BLOCK_WEIGHTS[self.format]


def head_dim_of(a: EncoderArch, layer: int) -> int:
    return a.head_dim if a.sliding[layer] else a.global_head_dim


def synthesize(arch: EncoderArch, seed: int = 0) -> dict:
    rng = np.random.default_rng(seed)
    a = arch

    def w(fmt, rows, cols):
        return W(fmt, rows, cols, synth.blocks(rng, fmt, rows, cols))

    def gain(n):
        return (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)

    m = {"arch": a, "token_embd": w(Q8_0, a.vocab, a.hidden), "output_norm": gain(a.hidden),
         "output": w(Q4_0, a.embedding, a.hidden), "per_layer_proj": w(Q4_0, a.layers * a.per_layer, a.hidden),
         "per_layer_norm": gain(a.per_layer), "layers": []}
    for l in range(a.layers):
        d = head_dim_of(a, l)
        qd, kvd = a.query_heads * d, a.kv_heads * d
        m["layers"].append({
            "attn_norm": gain(a.hidden), "q": w(Q4_0, qd, a.hidden), "k": w(Q4_0, kvd, a.hidden),
            "v": w(Q4_0, kvd, a.hidden), "q_norm": gain(d), "k_norm": gain(d),
            "o": w(Q4_0, a.hidden, qd), "post_attn_norm": gain(a.hidden), "ffn_norm": gain(a.hidden),
            "gate": w(Q4_0, a.ffn, a.hidden), "up": w(Q4_0, a.ffn, a.hidden), "down": w(Q4_0, a.hidden, a.ffn),
            "post_ffn_norm": gain(a.hidden), "inp_gate": w(Q4_0, a.per_layer, a.hidden),
            "proj": w(Q4_0, a.hidden, a.per_layer), "post_norm": gain(a.hidden),
            "output_scale": np.array([0.5 + rng.random()], np.float32)})
    return m


def _bools(key, items):
    return _kv(key, ARRAY, struct.pack("<IQ", BOOL, len(items)) + bytes(int(b) for b in items))


def write_gguf(m: dict, path: str) -> None:
    a = m["arch"]
    k = lambda s: f"{ARCH}.{s}"   # noqa: E731
    md = [_str("general.architecture", ARCH), _u32("general.alignment", ALIGNMENT),
          _u32(k("block_count"), a.layers), _u32(k("context_length"), a.context),
          _u32(k("embedding_length"), a.hidden), _u32(k("feed_forward_length"), a.ffn),
          _u32(k("attention.head_count"), a.query_heads), _u32(k("attention.head_count_kv"), a.kv_heads),
          _u32(k("attention.key_length"), a.global_head_dim), _u32(k("attention.value_length"), a.global_head_dim),
          _f32(k("attention.layer_norm_rms_epsilon"), a.epsilon), _f32(k("rope.freq_base"), a.rope_base),
          _kv(k("attention.causal"), BOOL, b"\x00"), _u32(k("pooling_type"), 1),
          _u32(k("attention.sliding_window"), a.window), _bools(k("attention.sliding_window_pattern"), a.sliding),
          _u32(k("attention.key_length_swa"), a.head_dim), _f32(k("rope.freq_base_swa"), a.swa_base),
          _u32(k("embedding_length_per_layer_input"), a.per_layer), _u32(k("embedding_length_out"), a.embedding),
          _strings("tokenizer.ggml.tokens", [f"t{i}" for i in range(a.vocab)])]
    ts = []

    def weight(name, x):
        ts.append((name, [x.cols, x.rows], x.format, np.ascontiguousarray(x.stored, np.uint8).tobytes()))

    def f32(name, g):
        ts.append((name, [g.size], T_F32, np.ascontiguousarray(g, np.float32).tobytes()))

    weight("token_embd.weight", m["token_embd"])
    f32("output_norm.weight", m["output_norm"])
    weight("output.weight", m["output"])
    weight("per_layer_model_proj.weight", m["per_layer_proj"])
    f32("per_layer_proj_norm.weight", m["per_layer_norm"])
    for i, L in enumerate(m["layers"]):
        p = f"blk.{i}."
        f32(p + "attn_norm.weight", L["attn_norm"])
        weight(p + "attn_q.weight", L["q"])
        weight(p + "attn_k.weight", L["k"])
        weight(p + "attn_v.weight", L["v"])
        f32(p + "attn_q_norm.weight", L["q_norm"])
        f32(p + "attn_k_norm.weight", L["k_norm"])
        weight(p + "attn_output.weight", L["o"])
        f32(p + "post_attention_norm.weight", L["post_attn_norm"])
        f32(p + "ffn_norm.weight", L["ffn_norm"])
        weight(p + "ffn_gate.weight", L["gate"])
        weight(p + "ffn_up.weight", L["up"])
        weight(p + "ffn_down.weight", L["down"])
        f32(p + "post_ffw_norm.weight", L["post_ffn_norm"])
        weight(p + "inp_gate.weight", L["inp_gate"])
        weight(p + "proj.weight", L["proj"])
        f32(p + "post_norm.weight", L["post_norm"])
        f32(p + "layer_output_scale.weight", L["output_scale"])
    head = b"GGUF" + struct.pack("<IQQ", 3, len(ts), len(md)) + b"".join(md)
    infos, offset = b"", 0
    for name, dims, ttype, data in ts:
        infos += _string(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        infos += struct.pack("<IQ", ttype, offset)
        offset += (len(data) + ALIGNMENT - 1) // ALIGNMENT * ALIGNMENT
    with open(path, "wb") as f:
        f.write(head + infos)
        f.write(b"\0" * ((-(len(head) + len(infos))) % ALIGNMENT))
        for _, _, _, data in ts:
            f.write(data)
            f.write(b"\0" * ((-len(data)) % ALIGNMENT))


def _mm(x: W, inp: np.ndarray) -> np.ndarray:
    return O.matmul(x.format, O.to_piece(x.format, x.stored), x.blocks, x.rows, x.cols, inp)


def _act(g: np.ndarray) -> np.ndarray:
    f = np.vectorize(lambda v: O.lib().or_activate(GELU_TANH, float(v)), otypes=[np.float32])
    return f(g).astype(np.float32)


def oracle_embedding(m: dict, ids) -> np.ndarray:
    """The unit-length embedding of one step of `ids` at position 0."""
    a = m["arch"]
    ids = list(ids)
    N, Wd, P = len(ids), a.hidden, a.per_layer
    eps = np.float32(a.epsilon)
    # embed: each row unpacked from the table, times √W in f32
    e = m["token_embd"]
    piece = O.to_piece(e.format, e.stored)
    scale = np.float32(math.sqrt(np.float32(Wd)))
    hidden = np.empty((N, Wd), np.float32)
    for t, i in enumerate(ids):
        for g in range(Wd // 32):
            hidden[t, 32 * g:32 * g + 32] = O.unpack(e.format, piece, e.blocks, i * (Wd // 32) + g) * scale
    # per-layer inputs: one product, then each P-wide slice normed with ε·W
    raw = _mm(m["per_layer_proj"], hidden)
    per_layer = np.empty_like(raw)
    eps_w = float(np.float32(eps * np.float32(Wd)))
    for t in range(N):
        for l in range(a.layers):
            _, per_layer[t, l * P:(l + 1) * P] = O.norm_row_ex(raw[t, l * P:(l + 1) * P], None, m["per_layer_norm"],
                                                               epsilon=eps_w, add=False)
    output = np.zeros((N, Wd), np.float32)
    normed = np.zeros((N, Wd), np.float32)
    pending = {"add": False, "post": None, "scale": None}

    def norm(gain, normalize=True):
        for t in range(N):
            h, n = O.norm_row_ex(hidden[t], output[t], gain, epsilon=float(eps), add=pending["add"],
                                 post_gain=pending["post"], scale=pending["scale"], normalize=normalize)
            hidden[t] = h
            if normalize:
                normed[t] = n

    for l, L in enumerate(m["layers"]):
        d = head_dim_of(a, l)
        # attention
        norm(L["attn_norm"])
        q, k, v = _mm(L["q"], normed), _mm(L["k"], normed), _mm(L["v"], normed)
        base = a.swa_base if a.sliding[l] else a.rope_base
        turns = O.rope_turns(base, d)
        for t in range(N):
            qt, kt, vt = q[t].copy(), k[t].copy(), v[t].copy()
            O.rope_encode_token(qt, kt, vt, t, head_dim=d, query_heads=a.query_heads, kv_heads=a.kv_heads,
                                halves=True, epsilon=float(eps), turns=turns, query_gain=L["q_norm"],
                                key_gain=L["k_norm"], value_norm=True)
            q[t], k[t], v[t] = qt, kt, vt
        window = a.window if a.sliding[l] else a.context
        att = O.block_attention(q, k, v, tokens=N, head_dim=d, query_heads=a.query_heads, kv_heads=a.kv_heads,
                                half_window=window // 2, scale_log2e=float(np.float32(1.4426950408889634)))
        output[:] = _mm(L["o"], att)
        pending = {"add": True, "post": L["post_attn_norm"], "scale": None}
        # gated feed-forward
        norm(L["ffn_norm"])
        act = (_act(_mm(L["gate"], normed)) * _mm(L["up"], normed)).astype(np.float32)
        output[:] = _mm(L["down"], act)
        pending = {"add": True, "post": L["post_ffn_norm"], "scale": None}
        # the per-layer block: the add alone, the gate by the layer's input, the projection
        norm(L["post_norm"], normalize=False)
        gated = (_act(_mm(L["inp_gate"], hidden)) * per_layer[:, l * P:(l + 1) * P]).astype(np.float32)
        output[:] = _mm(L["proj"], gated)
        pending = {"add": True, "post": L["post_norm"], "scale": L["output_scale"]}
    norm(m["output_norm"])
    pooled = O.pool_mean(normed)
    projected = _mm(m["output"], pooled[None, :])[0]
    return O.pool_unit(projected)
