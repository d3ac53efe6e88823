"""Batched decode over several GPUs: sequences sharded over ranks, and the
large-vocabulary head split by vocabulary with one exchange of candidates.

Each rank holds `sequences / world` sequences in a BatchDecoder (its own
caches, no exchange for the layers). For the head, every rank needs every
sequence's final hidden row, so the normed rows are all-gathered first; then
rank r computes the logits of vocabulary rows [v0_r, v1_r) for all rows
(an exact product: each logit's bits are those of the whole-vocabulary
product), keeps each row's top 64 of its shard under the reference's total
order with global token ids (cb_select_run, candidates_only), and the
candidate lists are all-gathered ([world][rows][64] pairs). The union of the
shards' top 64 holds the whole vocabulary's top 64, so the merge
(cb_select_merge_run, the same on every rank) gives exactly the candidates —
and the draw — of one selection over the whole vocabulary. Each rank writes
its own rows' records back into its decoder, which feeds the next step.

The collectives go through torch.distributed (NCCL between GPUs) on the
decoder's CUDA stream; `collective` may be replaced (tests emulate several
ranks on one device by running the shards in turn)."""
from __future__ import annotations

import ctypes

import numpy as np

import charlotte_b200 as cb
from charlotte_b200 import model as M

KEEP = 64   # candidates a row keeps (topk.wgsl)


def shard_rows(vocab: int, world: int, rank: int) -> tuple[int, int]:
    """Vocabulary rows [v0, v1) of a rank: contiguous, as even as whole rows allow."""
    return vocab * rank // world, vocab * (rank + 1) // world


class _Raw:
    """A device pointer as a torch tensor (via __cuda_array_interface__)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3, "strides": None}


def device_view(ptr: int, shape, dtype):
    import torch
    typestr = {torch.float32: "<f4", torch.int32: "<i4"}[dtype]
    return torch.as_tensor(_Raw(ptr, shape, typestr), device="cuda")


class _Ptr:
    """A raw device pointer where the bindings take a tensor."""

    def __init__(self, ptr: int):
        self.ptr = int(ptr)

    def data_ptr(self) -> int:
        return self.ptr


class SplitHead:
    """The vocabulary shard of one rank's head and its buffers for `rows`
    sequences in all (every rank's)."""

    def __init__(self, dec: M.BatchDecoder, rows: int, world: int, rank: int):
        import torch
        L = dec.lib
        for name, res, args in (("cb_decoder_stream", ctypes.c_void_p, [ctypes.c_void_p]),
                                ("cb_decoder_device_normed", ctypes.c_void_p, [ctypes.c_void_p]),
                                ("cb_decoder_device_sampled", ctypes.c_void_p, [ctypes.c_void_p]),
                                ("cb_decoder_step_body", ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p,
                                                                        ctypes.c_uint32])):
            getattr(L, name).restype = res
            getattr(L, name).argtypes = args
        L.cb_decoder_head.restype = ctypes.c_int
        L.cb_decoder_head.argtypes = [ctypes.c_void_p, ctypes.POINTER(cb.Member), ctypes.POINTER(ctypes.c_uint32),
                                      ctypes.POINTER(ctypes.c_uint32)]
        self.dec, self.rows, self.world, self.rank = dec, rows, world, rank
        member, fmt, cols = cb.Member(), ctypes.c_uint32(), ctypes.c_uint32()
        M._check(L.cb_decoder_head(dec.handle, ctypes.byref(member), ctypes.byref(fmt), ctypes.byref(cols)))
        self.fmt, self.hidden = fmt.value, cols.value
        self.vocab = member.rows
        self.v0, self.v1 = shard_rows(self.vocab, world, rank)
        self.head = (_Ptr(member.piece), member.blocks, self.v0, self.v1 - self.v0, 0)
        self.stream = torch.cuda.ExternalStream(L.cb_decoder_stream(dec.handle))
        self.local = dec.sequences
        n = self.v1 - self.v0
        tiles = cb.lib().cb_select_tiles(n)
        with torch.cuda.stream(self.stream):
            self.normed_all = torch.empty((rows, self.hidden), dtype=torch.float32, device="cuda")
            self.logits = torch.empty((rows, n), dtype=torch.float32, device="cuda")
            self.partials = torch.empty(rows * tiles * 2 * KEEP, dtype=torch.int32, device="cuda")
            self.ticket = torch.zeros(rows * cb.lib().cb_select_tickets(n), dtype=torch.int32, device="cuda")
            self.cand = torch.empty((rows, 2 * KEEP), dtype=torch.int32, device="cuda")
            self.cand_all = torch.empty((world, rows, 2 * KEEP), dtype=torch.int32, device="cuda")
            self.merged = torch.empty((rows, 2 * KEEP), dtype=torch.int32, device="cuda")
            self.sampled_all = torch.empty((rows, 4), dtype=torch.int32, device="cuda")

    def local_normed(self):
        return device_view(self.dec.lib.cb_decoder_device_normed(self.dec.handle), (self.local, self.hidden),
                           __import__("torch").float32)

    def local_sampled(self):
        return device_view(self.dec.lib.cb_decoder_device_sampled(self.dec.handle), (self.local, 4),
                           __import__("torch").int32)

    def body(self, position: int, ids=None):
        """The batched step up to the final norm (fed from the last records
        when ids is None)."""
        ptr = None
        if ids is not None:
            ids = np.ascontiguousarray(ids, np.uint32)
            ptr = ids.ctypes.data
        M._check(self.dec.lib.cb_decoder_step_body(self.dec.handle, ptr, position))

    def shard_candidates(self):
        """This rank's shard of the head for every row, and each row's top 64
        of it with global ids, into self.cand (after normed_all is filled)."""
        import torch
        with torch.cuda.stream(self.stream):
            n = self.v1 - self.v0
            cb.matmul(self.fmt, self.hidden, [self.head], self.normed_all, [self.logits], stream=self.stream)
            cb.run("select", logits=self.logits, count=n, partials=self.partials, ticket=self.ticket,
                   candidates=self.cand, sampled=None, rows=self.rows, logits_stride=n, id_offset=self.v0,
                   candidates_only=1, stream=self.stream)

    def merge(self, position: int, sampling: M.CSampling | None = None):
        """Every rank's candidate lists (self.cand_all) merged and drawn; this
        rank's rows' records written back into its decoder."""
        import math
        import torch
        s = sampling or M.Decoder.sampling()
        with torch.cuda.stream(self.stream):
            cb.run("select_merge", lists_data=self.cand_all, lists=self.world, rows=self.rows,
                   candidates=self.merged, sampled=self.sampled_all, position=None, position0=position, tokens=1,
                   seed0=s.seed0, seed1=s.seed1, top_k=s.top_k or 1, temperature=s.temperature, top_p=s.top_p,
                   min_p=s.min_p, log_min_p=math.log(s.min_p) if s.min_p > 0 else 0.0, stream=self.stream)
            mine = self.sampled_all[self.rank * self.local:(self.rank + 1) * self.local]
            self.local_sampled().copy_(mine)

    def step(self, position: int, ids=None, sampling=None, timing=None):
        """One batched step across ranks through torch.distributed. With
        `timing` (a list), CUDA events around the two all-gathers on the
        decoder's stream are appended to it: (before rows, after rows,
        before candidates, after candidates)."""
        import torch
        import torch.distributed as dist
        self.body(position, ids)
        events = [torch.cuda.Event(enable_timing=True) for _ in range(4)] if timing is not None else None
        with torch.cuda.stream(self.stream):
            if events:
                events[0].record(self.stream)
            dist.all_gather_into_tensor(self.normed_all, self.local_normed().contiguous())
            if events:
                events[1].record(self.stream)
            self.shard_candidates()
            if events:
                events[2].record(self.stream)
            dist.all_gather_into_tensor(self.cand_all, self.cand)
            if events:
                events[3].record(self.stream)
            self.merge(position, sampling)
        if events:
            timing.append(events)
        return self.sampled_all
