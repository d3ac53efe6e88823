"""charlotte_b200: a B200 (sm_100a) CUDA backend for the hot path of Charlotte
(plainsight-systems/charlotte) — GGUF dequant-matmul, RMSNorm, QK-norm + RoPE
+ KV append, chunked attention, gather, top-k and the draw — behind a C ABI
(include/charlotte_b200.h).

This module is the host-side binding of that C ABI (ctypes over
libcharlotte_b200.so), taking torch CUDA tensors for device memory and
streams. There is no CPU path: every call runs the CUDA kernels, and loading
fails loudly when the library is missing.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libcharlotte_b200.so")

F32, F16, Q4_0, Q4_1, Q8_0, Q6_K, BF16 = 0, 1, 2, 3, 8, 14, 30
WRITE, QKV, GATED, GATED_BY_INPUT = 0, 1, 2, 3
SILU, GELU_TANH, SIGMOID = 0, 1, 2
MATMUL_PDL, MATMUL_TENSOR, MATMUL_STREAMED, MATMUL_TILED, MATMUL_SPLIT = 1, 2, 4, 8, 16
OK, ERROR_BUILD, ERROR_STEP, ERROR_DEVICE_LOST, ERROR_CANCELLED, ERROR_INVALID = range(6)


class CharlotteError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"[status {status}] {message}")
        self.status = status


class Member(ctypes.Structure):
    _fields_ = [("piece", ctypes.c_void_p), ("blocks", ctypes.c_uint32), ("first_row", ctypes.c_uint32),
                ("rows", ctypes.c_uint32), ("out_offset", ctypes.c_uint32)]


class Matmul(ctypes.Structure):
    _fields_ = [("format", ctypes.c_uint32), ("columns", ctypes.c_uint32), ("members", ctypes.c_uint32),
                ("epilogue", ctypes.c_uint32), ("activation", ctypes.c_uint32), ("member", Member * 3),
                ("gate_input", ctypes.c_void_p), ("gate_input_stride", ctypes.c_uint32),
                ("gate_input_column", ctypes.c_uint32), ("gate_input_token", ctypes.c_uint32),
                ("scratch", ctypes.c_void_p), ("scratch_bytes", ctypes.c_uint64), ("dense", ctypes.c_void_p),
                ("x16", ctypes.c_void_p), ("out16", ctypes.c_void_p)]


class Norm(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_void_p), ("output", ctypes.c_void_p), ("gain", ctypes.c_void_p),
                ("post_gain", ctypes.c_void_p), ("normed", ctypes.c_void_p), ("width", ctypes.c_uint32),
                ("tokens", ctypes.c_uint32), ("add", ctypes.c_uint32), ("last_token", ctypes.c_uint32),
                ("epsilon", ctypes.c_float), ("scale", ctypes.c_void_p), ("add_only", ctypes.c_uint32),
                ("rows_per_token", ctypes.c_uint32), ("normed16", ctypes.c_void_p)]


class Rope(ctypes.Structure):
    _fields_ = [("query", ctypes.c_void_p), ("key", ctypes.c_void_p), ("value", ctypes.c_void_p),
                ("key_cache", ctypes.c_void_p), ("value_cache", ctypes.c_void_p), ("query_gain", ctypes.c_void_p),
                ("key_gain", ctypes.c_void_p), ("factors", ctypes.c_void_p), ("turns", ctypes.c_void_p),
                ("position", ctypes.c_void_p), ("position0", ctypes.c_uint32), ("tokens", ctypes.c_uint32),
                ("head_dim", ctypes.c_uint32), ("query_heads", ctypes.c_uint32), ("kv_heads", ctypes.c_uint32),
                ("halves", ctypes.c_uint32), ("slots", ctypes.c_uint32), ("epsilon", ctypes.c_float),
                ("rows_are_sequences", ctypes.c_uint32), ("sequence_stride", ctypes.c_uint64),
                ("encode", ctypes.c_uint32), ("value_norm", ctypes.c_uint32)]


class BlockAttention(ctypes.Structure):
    _fields_ = [("query", ctypes.c_void_p), ("key", ctypes.c_void_p), ("value", ctypes.c_void_p),
                ("out", ctypes.c_void_p), ("tokens", ctypes.c_uint32), ("head_dim", ctypes.c_uint32),
                ("query_heads", ctypes.c_uint32), ("kv_heads", ctypes.c_uint32), ("half_window", ctypes.c_uint32),
                ("scale_log2e", ctypes.c_float)]


class Pool(ctypes.Structure):
    _fields_ = [("input", ctypes.c_void_p), ("output", ctypes.c_void_p), ("width", ctypes.c_uint32),
                ("tokens", ctypes.c_uint32), ("kind", ctypes.c_uint32)]


POOL_MEAN, POOL_UNIT = 0, 1


class Attention(ctypes.Structure):
    _fields_ = [("query", ctypes.c_void_p), ("key_cache", ctypes.c_void_p), ("value_cache", ctypes.c_void_p),
                ("out", ctypes.c_void_p), ("partials", ctypes.c_void_p), ("stats", ctypes.c_void_p),
                ("tickets", ctypes.c_void_p), ("position", ctypes.c_void_p), ("position0", ctypes.c_uint32),
                ("tokens", ctypes.c_uint32), ("head_dim", ctypes.c_uint32), ("query_heads", ctypes.c_uint32),
                ("kv_heads", ctypes.c_uint32), ("slots", ctypes.c_uint32), ("window", ctypes.c_uint32),
                ("max_chunks", ctypes.c_uint32), ("scale_log2e", ctypes.c_float),
                ("rows_are_sequences", ctypes.c_uint32), ("sequence_stride", ctypes.c_uint64),
                ("rope", ctypes.c_void_p), ("out16", ctypes.c_void_p)]


class Gather(ctypes.Structure):
    _fields_ = [("piece", ctypes.c_void_p), ("format", ctypes.c_uint32), ("blocks", ctypes.c_uint32),
                ("width", ctypes.c_uint32), ("first_row", ctypes.c_uint32), ("row_count", ctypes.c_uint32),
                ("ids", ctypes.c_void_p), ("sampled", ctypes.c_void_p), ("fed", ctypes.c_uint32),
                ("tokens", ctypes.c_uint32), ("scale", ctypes.c_float), ("hidden", ctypes.c_void_p),
                ("fed_stride", ctypes.c_uint32)]


class Select(ctypes.Structure):
    _fields_ = [("logits", ctypes.c_void_p), ("count", ctypes.c_uint32), ("partials", ctypes.c_void_p),
                ("ticket", ctypes.c_void_p), ("candidates", ctypes.c_void_p), ("sampled", ctypes.c_void_p),
                ("position", ctypes.c_void_p), ("position0", ctypes.c_uint32), ("tokens", ctypes.c_uint32),
                ("seed0", ctypes.c_uint32), ("seed1", ctypes.c_uint32), ("top_k", ctypes.c_uint32),
                ("temperature", ctypes.c_float), ("top_p", ctypes.c_float), ("min_p", ctypes.c_float),
                ("log_min_p", ctypes.c_float), ("rows", ctypes.c_uint32), ("logits_stride", ctypes.c_uint32),
                ("id_offset", ctypes.c_uint32), ("candidates_only", ctypes.c_uint32)]


class SelectMerge(ctypes.Structure):
    _fields_ = [("lists_data", ctypes.c_void_p), ("lists", ctypes.c_uint32), ("rows", ctypes.c_uint32),
                ("candidates", ctypes.c_void_p), ("sampled", ctypes.c_void_p), ("position", ctypes.c_void_p),
                ("position0", ctypes.c_uint32), ("tokens", ctypes.c_uint32), ("seed0", ctypes.c_uint32),
                ("seed1", ctypes.c_uint32), ("top_k", ctypes.c_uint32), ("temperature", ctypes.c_float),
                ("top_p", ctypes.c_float), ("min_p", ctypes.c_float), ("log_min_p", ctypes.c_float)]


RUN_PDL = 1
RUN_TENSOR = 2   # cb_attention_run: the tensor-core form (tolerance tier)
_lib = None


def library_path() -> str:
    return LIB_PATH


def lib() -> ctypes.CDLL:
    """The loaded C ABI library. Raises when it has not been built: there is
    no fallback."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m charlotte_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        L.cb_last_error.restype = ctypes.c_size_t
        L.cb_last_error.argtypes = [ctypes.c_char_p, ctypes.c_size_t]
        L.cb_version.restype = ctypes.c_char_p
        L.cb_device_sm_count.restype = ctypes.c_int
        L.cb_fault_check.restype = ctypes.c_int
        L.cb_fault_check.argtypes = [ctypes.POINTER(ctypes.c_uint)]
        L.cb_debug_spin_limit.restype = ctypes.c_int
        L.cb_debug_spin_limit.argtypes = [ctypes.c_int32]
        L.cb_matmul_run.restype = ctypes.c_int
        L.cb_matmul_run.argtypes = [ctypes.POINTER(Matmul), ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32,
                                    ctypes.POINTER(ctypes.c_void_p * 3), ctypes.POINTER(ctypes.c_uint32 * 3),
                                    ctypes.c_uint32, ctypes.c_void_p]
        for name, struct in (("cb_norm_run", Norm), ("cb_rope_run", Rope), ("cb_attention_run", Attention),
                             ("cb_block_attention_run", BlockAttention), ("cb_pool_run", Pool),
                             ("cb_gather_run", Gather), ("cb_select_run", Select),
                             ("cb_select_run_static", Select), ("cb_select_merge_run", SelectMerge)):
            fn = getattr(L, name)
            fn.restype = ctypes.c_int
            fn.argtypes = [ctypes.POINTER(struct), ctypes.c_uint32, ctypes.c_void_p]
        L.cb_rope_turns.argtypes = [ctypes.c_double, ctypes.c_uint32, ctypes.POINTER(ctypes.c_float)]
        L.cb_attention_tickets.restype = ctypes.c_uint32
        L.cb_attention_tickets.argtypes = [ctypes.c_uint32] * 3
        L.cb_select_tiles.restype = ctypes.c_uint32
        L.cb_select_tiles.argtypes = [ctypes.c_uint32]
        L.cb_select_tickets.restype = ctypes.c_uint32
        L.cb_select_tickets.argtypes = [ctypes.c_uint32]
        L.cb_matmul_scratch_bytes.restype = ctypes.c_uint64
        L.cb_matmul_scratch_bytes.argtypes = [ctypes.c_uint32] * 3
        L.cb_matmul_split_bytes.restype = ctypes.c_uint64
        L.cb_matmul_split_bytes.argtypes = [ctypes.c_uint32] * 2
        L.cb_matmul_dense_bytes.restype = ctypes.c_uint64
        L.cb_matmul_dense_bytes.argtypes = [ctypes.POINTER(Matmul)]
        L.cb_matmul_densify.restype = ctypes.c_int
        L.cb_matmul_densify.argtypes = [ctypes.POINTER(Matmul), ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p]
        _lib = L
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    lib().cb_last_error(buf, 1024)
    return buf.value.decode(errors="replace")


def check(status: int) -> None:
    if status != OK:
        raise CharlotteError(status, last_error())


def _stream(stream) -> int:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


def _product(fmt, columns, members, epilogue, activation) -> "Matmul":
    m = Matmul()
    m.format = fmt
    m.columns = columns
    m.members = len(members)
    m.epilogue = epilogue
    m.activation = activation
    for i, (piece, blocks, first_row, rows, out_offset) in enumerate(members):
        m.member[i] = Member(piece.data_ptr(), blocks, first_row, rows, out_offset)
    return m


def densify(fmt: int, columns: int, members, *, epilogue: int = WRITE, activation: int = SILU, stream=None):
    """cb_matmul_densify: the product's weights as f16 rows in the dense
    form's slot order (a uint8 cuda tensor), for matmul(..., dense=)."""
    import torch
    m = _product(fmt, columns, members, epilogue, activation)
    n = lib().cb_matmul_dense_bytes(ctypes.byref(m))
    if n == 0:
        raise CharlotteError(ERROR_INVALID, last_error())
    out = torch.empty(n, dtype=torch.uint8, device=members[0][0].device)
    check(lib().cb_matmul_densify(ctypes.byref(m), out.data_ptr(), n, _stream(stream)))
    return out


def matmul(fmt: int, columns: int, members, x, out, *, epilogue: int = WRITE, activation: int = SILU,
           tokens: int | None = None, x_stride: int | None = None, out_stride=None, flags: int = 0,
           gate_input=None, gate_input_stride: int = 0, gate_input_column: int = 0, gate_input_token: int = 0,
           stream=None, scratch=None, dense=None) -> None:
    """Runs cb_matmul_run. `members`: list of (piece tensor (uint8, cuda), blocks,
    first_row, rows, out_offset). `x`: f32 cuda tensor [tokens, x_stride].
    `out`: list of up to 3 f32 cuda tensors. With MATMUL_TENSOR, `scratch`
    (a cuda tensor of cb_matmul_scratch_bytes) or one allocated here, and
    `dense` (densify's tensor for the same product) for the dense form."""
    m = _product(fmt, columns, members, epilogue, activation)
    m.dense = _ptr(dense)
    m.gate_input = _ptr(gate_input)
    m.gate_input_stride = gate_input_stride
    m.gate_input_column = gate_input_column
    m.gate_input_token = gate_input_token
    if tokens is None:
        tokens = x.shape[0] if x.dim() > 1 else 1
    if x_stride is None:
        x_stride = x.shape[-1]
    if flags & MATMUL_TENSOR and scratch is None:
        need = lib().cb_matmul_scratch_bytes(flags, tokens, columns)
        import torch
        scratch = torch.empty(need, dtype=torch.uint8, device=x.device)
    if scratch is not None:   # the tensor form's x16, or the split form's range sums
        m.scratch = scratch.data_ptr()
        m.scratch_bytes = scratch.numel() * scratch.element_size()
    outs = (ctypes.c_void_p * 3)(*[_ptr(o) for o in (list(out) + [None, None, None])[:3]])
    if out_stride is None:
        out_stride = [o.shape[-1] if o is not None else 0 for o in (list(out) + [None, None, None])[:3]]
    strides = (ctypes.c_uint32 * 3)(*out_stride)
    check(lib().cb_matmul_run(ctypes.byref(m), x.data_ptr(), x_stride, tokens, ctypes.byref(outs),
                              ctypes.byref(strides), flags, _stream(stream)))


def run(entry: str, **fields) -> None:
    """Runs one kernel entry point: `entry` in norm, rope, attention, gather,
    select, select_static, select_merge, block_attention, pool; fields are the
    C struct's (tensors become device pointers)."""
    struct = {"norm": Norm, "rope": Rope, "attention": Attention, "gather": Gather, "select": Select,
              "select_static": Select, "select_merge": SelectMerge, "block_attention": BlockAttention,
              "pool": Pool}[entry]
    fn = {"select_static": "cb_select_run_static"}.get(entry, f"cb_{entry}_run")
    stream = fields.pop("stream", None)
    flags = fields.pop("flags", 0)
    v = struct()
    keep = []   # nested structs, alive through the call
    for name, value in fields.items():
        if isinstance(value, dict):   # attention's fused rope: a cb_rope passed by pointer
            sub = Rope()
            for n2, v2 in value.items():
                setattr(sub, n2, v2.data_ptr() if hasattr(v2, "data_ptr") else v2)
            keep.append(sub)
            value = ctypes.addressof(sub)
        if hasattr(value, "data_ptr"):
            value = value.data_ptr()
        setattr(v, name, value)
    check(getattr(lib(), fn)(ctypes.byref(v), flags, _stream(stream)))


def rope_turns(base: float, head_dim: int):
    import numpy as np
    t = np.empty(head_dim // 2, np.float32)
    lib().cb_rope_turns(base, head_dim, t.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    return t
