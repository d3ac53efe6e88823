"""The drop-in boundary end to end: a model file loaded and stepped the way
the reference's runtime does it — its GGUF reader, architecture
description, residency plan, upload routes and piece writer, and the
decoder graph its launchers describe (kernels::Launch), all the reference's
own code compiled into integration/libcharlotte_program.so — with the CUDA
Upload and Program (integration/program_cuda.h over cb_buffers and
cb_program) in place of the WebGPU ones.

Parity: every step's record (the draw's 16 bytes) and the logits equal the
oracle's pass over the same weights bit for bit, and equal the C ABI
decoder's; steps run pipelined (the next fed step enqueued before the last
one's readback is delivered, at most two outstanding), and their records
arrive in run order (src/core/kernels/program.h:62-70, order.h:30)."""
import ctypes
import os

import numpy as np
import pytest

import charlotte_b200 as cb
from charlotte_b200 import model as M
from gguf_writer import write as write_gguf

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "integration", "libcharlotte_program.so")


class Harness:
    def __init__(self, path, max_chunk=1 << 16):
        cb.lib()   # libcharlotte_b200 first: the harness links it
        assert os.path.exists(LIB), "integration/libcharlotte_program.so is missing: the boundary cannot be tested"
        L = ctypes.CDLL(LIB)
        L.cbh_open.restype = ctypes.c_int
        L.cbh_open.argtypes = [ctypes.c_char_p, ctypes.c_uint32, ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p,
                               ctypes.c_size_t]
        for name in ("cbh_vocab", "cbh_launches", "cbh_context", "cbh_outstanding"):
            getattr(L, name).restype = ctypes.c_uint32
            getattr(L, name).argtypes = [ctypes.c_void_p]
        L.cbh_run.restype = ctypes.c_int
        L.cbh_run.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                              ctypes.c_uint32, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                              ctypes.c_uint32]
        L.cbh_poll.restype = ctypes.c_int
        L.cbh_poll.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_uint32]
        L.cbh_logits.restype = ctypes.c_int
        L.cbh_logits.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        L.cbh_message.restype = ctypes.c_char_p
        L.cbh_message.argtypes = [ctypes.c_void_p]
        L.cbh_profile.restype = ctypes.c_int
        L.cbh_profile.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                  ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32,
                                  ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_int32)]
        L.cbh_close.argtypes = [ctypes.c_void_p]
        self.L = L
        h = ctypes.c_void_p()
        err = ctypes.create_string_buffer(1024)
        rc = L.cbh_open(path.encode(), max_chunk, ctypes.byref(h), err, 1024)
        assert rc == 0, err.value.decode()
        self.h = h
        self.vocab = L.cbh_vocab(h)
        self.launches = L.cbh_launches(h)

    def run(self, ids, position, logits=True, fed=False, tag=0, sampling=None, top_k=1, seed=(0, 0)):
        ids = np.ascontiguousarray(ids if ids is not None else [0], np.uint32)
        smp = np.asarray(sampling, np.float32) if sampling is not None else None
        self.L.cbh_run(self.h, ids.ctypes.data, ids.size, position, int(logits), int(fed),
                       smp.ctypes.data if smp is not None else None, top_k, seed[0], seed[1], tag)

    def poll(self, wait=True):
        out = np.zeros((8, 6), np.uint32)
        n = self.L.cbh_poll(self.h, int(wait), out.ctypes.data, 8)
        return out[:n]

    def drain(self):
        got = []
        while self.L.cbh_outstanding(self.h):
            got += list(self.poll(wait=True))
        return np.array(got, np.uint32).reshape(-1, 6)

    def step(self, ids, position, logits=True, fed=False):
        self.run(ids, position, logits, fed)
        r = self.poll()
        assert len(r) == 1 and r[0, 1] == 0, (r, self.L.cbh_message(self.h))
        return r[0, 2:6].copy()

    def logits(self):
        out = np.empty(self.vocab, np.float32)
        assert self.L.cbh_logits(self.h, out.ctypes.data) == 0
        return out

    def close(self):
        if self.h:
            self.L.cbh_close(self.h)
            self.h = None


def _model(kind, tmp_path, seed):
    m = M.synthesize(M.tiny(kind), seed=seed)
    path = str(tmp_path / f"{kind}.gguf")
    write_gguf(m, path)
    return m, path


@pytest.mark.parametrize("kind", ["qwen3", "llama", "gemma3"])
def test_reference_graph_on_the_cuda_program_matches_the_oracle(cuda, tmp_path, kind):
    """The prompt in uneven steps (the reference's tile widths 8, 16 and 32
    all run), then 12 fed greedy steps pipelined two deep: records and the
    last logits equal the oracle's and the C ABI decoder's bit for bit."""
    from oracle.model import OracleDecoder
    m, path = _model(kind, tmp_path, seed=hash(kind) % 997)
    rng = np.random.default_rng(3)
    prompt = rng.integers(0, m.arch.vocab, 40).astype(np.uint32)
    h = Harness(path)
    at, rec = 0, None
    for n in (5, 12, 23):
        rec = h.step(prompt[at: at + n], at, logits=(at + n == prompt.size))
        at += n
    first_logits = h.logits()
    od = OracleDecoder(m)
    orec, olg = od.step(prompt, 0)
    np.testing.assert_array_equal(rec, orec)
    np.testing.assert_array_equal(first_logits, olg)
    # fed decode steps, the next one enqueued before the last one's record is read
    steps = 12
    records = []
    for i in range(steps):
        if h.L.cbh_outstanding(h.h) == 2:   # one running, one queued: wait for the oldest
            records += list(h.poll(wait=True))
        h.run(None, 40 + i, fed=True, tag=i)
        assert h.L.cbh_outstanding(h.h) <= 2
        records += list(h.poll(wait=False))
    records += list(h.drain())
    assert [int(r[0]) for r in records] == list(range(steps)), "records out of run order"
    assert all(int(r[1]) == 0 for r in records)
    want, prev = [], orec[0]
    for i in range(steps):
        r, lg = od.step([prev], 40 + i)
        want.append(int(r[0]))
        prev = r[0]
    assert [int(r[2]) for r in records] == want
    np.testing.assert_array_equal(h.logits(), lg)
    # the C ABI decoder, over the same model, agrees token for token
    dec = M.Decoder(m, max_step_tokens=64)
    dec.prefill(prompt)
    toks, _ = dec.generate(steps)
    assert toks.tolist() == want
    dec.close()
    od.close()
    h.close()


def test_third_outstanding_step_is_refused_and_late_positions_fail_unrun(cuda, tmp_path):
    m, path = _model("qwen3", tmp_path, seed=4)
    h = Harness(path)
    h.step(np.arange(8, dtype=np.uint32), 0)
    h.run(None, 8, fed=True, tag=1)
    h.run(None, 9, fed=True, tag=2)
    h.run(None, 10, fed=True, tag=3)   # a third while two are outstanding
    got = np.concatenate([h.poll(wait=False), h.drain()])
    tags = [int(r[0]) for r in got]
    # the refusal fires at once (first), then the two steps in run order
    assert tags == [3, 1, 2], tags
    assert int(got[0, 1]) == cb.ERROR_STEP and int(got[1, 1]) == 0 and int(got[2, 1]) == 0
    h.run(np.array([1], np.uint32), (1 << 24) - 1 + 1, tag=9)   # past position 2^24
    bad = h.drain()
    assert int(bad[0, 1]) == cb.ERROR_STEP
    # the program still steps afterwards
    h.step(np.array([2], np.uint32), 10)
    h.close()


def test_profiled_step_times_its_launches(cuda, tmp_path):
    m, path = _model("qwen3", tmp_path, seed=6)
    h = Harness(path)
    ids = np.arange(16, dtype=np.uint32)
    idx = np.zeros(4096, np.uint32)
    ends = np.zeros(4096, np.uint64)
    step_ns = ctypes.c_uint64()
    status = ctypes.c_int32()
    n = h.L.cbh_profile(h.h, ids.ctypes.data, ids.size, 0, 1, h.launches, idx.ctypes.data, ends.ctypes.data, 4096,
                        ctypes.byref(step_ns), ctypes.byref(status))
    assert status.value == 0 and n > 10
    assert np.all(np.diff(idx[:n].astype(np.int64)) > 0) and idx[n - 1] < h.launches
    assert np.all(np.diff(ends[:n].astype(np.int64)) >= 0) and 0 < ends[n - 1] <= step_ns.value
    # a prefix of the graph: fewer launches timed, nothing read back
    k = h.L.cbh_profile(h.h, ids.ctypes.data, ids.size, 0, 1, int(idx[n // 2]), idx.ctypes.data, ends.ctypes.data,
                        4096, ctypes.byref(step_ns), ctypes.byref(status))
    assert status.value == 0 and 0 < k < n
    h.close()
