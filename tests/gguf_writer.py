"""Writes a synthetic model (charlotte_b200.model.Model) as a GGUF v3 file —
TEST INFRASTRUCTURE: the integration tests load it through the reference's
own reader, description, plan and upload path (integration/), so the same
weights reach both that path and the C ABI decoder.

GGUF v3 (the published llama.cpp container): magic, version, tensor count,
metadata count, the metadata key/values, the tensor infos (name, dimensions
innermost first, type, offset from the data section), padding to the
alignment, then each tensor's stored blocks at its aligned offset. The
metadata keys are the ones the reference's descriptions read for the three
families (src/core/arch/describe.cpp:133-214, gemma3.cpp:30-57)."""
from __future__ import annotations

import struct

import numpy as np

U32, F32, STRING, ARRAY = 4, 6, 8, 9
ALIGNMENT = 32
T_F32 = 0


def _string(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _kv(key: str, vtype: int, payload: bytes) -> bytes:
    return _string(key) + struct.pack("<I", vtype) + payload


def _u32(key, v):
    return _kv(key, U32, struct.pack("<I", v))


def _f32(key, v):
    return _kv(key, F32, struct.pack("<f", v))


def _str(key, v):
    return _kv(key, STRING, _string(v))


def _strings(key, items):
    return _kv(key, ARRAY, struct.pack("<IQ", STRING, len(items)) + b"".join(_string(s) for s in items))


def metadata_of(model) -> list[bytes]:
    a = model.arch
    fam = family(a)
    md = [_str("general.architecture", fam), _u32("general.alignment", ALIGNMENT),
          _u32(f"{fam}.block_count", a.layers), _u32(f"{fam}.context_length", a.context),
          _u32(f"{fam}.embedding_length", a.hidden), _u32(f"{fam}.feed_forward_length", a.ffn),
          _u32(f"{fam}.attention.head_count", a.query_heads), _u32(f"{fam}.attention.head_count_kv", a.kv_heads),
          _u32(f"{fam}.attention.key_length", a.head_dim), _u32(f"{fam}.attention.value_length", a.head_dim),
          _f32(f"{fam}.attention.layer_norm_rms_epsilon", a.epsilon), _f32(f"{fam}.rope.freq_base", a.rope_base),
          _strings("tokenizer.ggml.tokens", [f"t{i}" for i in range(a.vocab)])]
    if a.window:
        md += [_u32("gemma3.attention.sliding_window", a.window),
               _u32("gemma3.attention.sliding_window_pattern", a.window_pattern),
               _f32("gemma3.rope.freq_base_swa", a.window_rope_base)]
    return md


def family(arch) -> str:
    if arch.post_norms:
        return "gemma3"
    if not arch.qk_norm:
        return "llama"
    return "qwen3"


def tensors_of(model) -> list[tuple[str, list[int], int, bytes]]:
    """(name, dimensions innermost first, GGUF type, stored bytes)."""
    out = []

    def weight(name, w):
        out.append((name, [w.cols, w.rows], w.format, np.ascontiguousarray(w.stored, np.uint8).tobytes()))

    def gain(name, g):
        if g is not None:
            out.append((name, [g.size], T_F32, np.ascontiguousarray(g, np.float32).tobytes()))

    weight("token_embd.weight", model.token_embd)
    gain("output_norm.weight", model.output_norm)
    if model.output is not None:
        weight("output.weight", model.output)
    if model.factors is not None:
        gain("rope_freqs.weight", model.factors)
    for i, L in enumerate(model.layers):
        p = f"blk.{i}."
        gain(p + "attn_norm.weight", L.attn_norm)
        weight(p + "attn_q.weight", L.q)
        weight(p + "attn_k.weight", L.k)
        weight(p + "attn_v.weight", L.v)
        gain(p + "attn_q_norm.weight", L.q_norm)
        gain(p + "attn_k_norm.weight", L.k_norm)
        weight(p + "attn_output.weight", L.o)
        gain(p + "post_attention_norm.weight", L.post_attn_norm)
        gain(p + "ffn_norm.weight", L.ffn_norm)
        weight(p + "ffn_gate.weight", L.gate)
        weight(p + "ffn_up.weight", L.up)
        weight(p + "ffn_down.weight", L.down)
        gain(p + "post_ffw_norm.weight", L.post_ffn_norm)
    return out


def write(model, path: str) -> None:
    md = metadata_of(model)
    ts = tensors_of(model)
    head = b"GGUF" + struct.pack("<IQQ", 3, len(ts), len(md)) + b"".join(md)
    infos, offset = b"", 0
    for name, dims, ttype, data in ts:
        infos += _string(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        infos += struct.pack("<IQ", ttype, offset)
        offset += (len(data) + ALIGNMENT - 1) // ALIGNMENT * ALIGNMENT
    with open(path, "wb") as f:
        f.write(head + infos)
        pos = len(head) + len(infos)
        f.write(b"\0" * ((-pos) % ALIGNMENT))
        for _, _, _, data in ts:
            f.write(data)
            f.write(b"\0" * ((-len(data)) % ALIGNMENT))
