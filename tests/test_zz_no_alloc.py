"""cb_select_run_static — top-k and the draw for callers that cannot
allocate device memory (their host plans every device byte up front, or
cudaMalloc is not allowed where they run) — against cb_select_run, the entry
point that takes caller-allocated scratch, and against the oracle's top-k and
draw. Through the C ABI, two calls in a row, each's candidates and sampled
record identical bit for bit (the tolerance every selection test here uses).

This file is collected last, so its tests run after every other test in the
same process; one test also runs the entry point in a fresh process, where
its first call is the one that looks up the scratch array's address."""
import math
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

import charlotte_b200 as cb
import oracle as O

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _select(kind, logits, position, **settings):
    count = logits.numel()
    cand = torch.zeros(128, dtype=torch.int32, device="cuda")
    rec = torch.zeros(4, dtype=torch.int32, device="cuda")
    scratch = {}
    if kind == "select":
        scratch = dict(partials=torch.zeros(cb.lib().cb_select_tiles(count) * 128, dtype=torch.int32, device="cuda"),
                       ticket=torch.zeros(cb.lib().cb_select_tickets(count), dtype=torch.int32, device="cuda"))
    min_p = settings.get("min_p", 0.0)
    cb.run(kind, logits=logits, count=count, candidates=cand, sampled=rec, position=0, position0=position, tokens=1,
           seed0=settings.get("seed0", 0), seed1=settings.get("seed1", 0), top_k=settings.get("top_k", 40),
           temperature=settings.get("temperature", 0.0), top_p=settings.get("top_p", 1.0), min_p=min_p,
           log_min_p=math.log(min_p) if min_p > 0 else 0.0, **scratch)
    torch.cuda.synchronize()
    cb.check(cb.lib().cb_fault_check(None))
    return cand.cpu().numpy().view(np.uint32), rec.cpu().numpy().view(np.uint32)


CALLS = [
    (151936, 10, dict(temperature=0.0, top_k=1)),                                   # greedy, Qwen3's vocabulary
    (262144, 11, dict(temperature=0.8, top_k=40, top_p=0.9, min_p=0.05, seed0=3)),  # the largest it holds
]


def test_static_scratch_matches_caller_scratch_and_oracle_twice_in_a_row(cuda):
    rng = np.random.default_rng(2026)
    for count, position, settings in CALLS:
        host = (rng.standard_normal(count) * 4).astype(np.float32)
        logits = torch.from_numpy(host).cuda()
        want_cand, want_rec = _select("select", logits, position, **settings)
        got_cand, got_rec = _select("select_static", logits, position, **settings)
        np.testing.assert_array_equal(got_cand, want_cand)
        np.testing.assert_array_equal(got_rec, want_rec)
        oracle_cand = O.topk64(host)
        np.testing.assert_array_equal(got_cand, oracle_cand)
        oracle_rec = O.draw(oracle_cand, position, 1, seed=(settings.get("seed0", 0), 0),
                            top_k=settings.get("top_k", 40), temperature=settings.get("temperature", 0.0),
                            top_p=settings.get("top_p", 1.0), min_p=settings.get("min_p", 0.0))
        np.testing.assert_array_equal(got_rec, oracle_rec)


def test_static_scratch_refuses_what_it_cannot_hold(cuda):
    logits = torch.zeros(262145, dtype=torch.float32, device="cuda")
    with pytest.raises(cb.CharlotteError) as e:
        _select("select_static", logits, 0)
    assert e.value.status == cb.ERROR_INVALID and "262" in str(e.value)


FRESH = r"""
import sys
sys.path.insert(0, {root!r})
import numpy as np, torch
import charlotte_b200 as cb
sys.path.insert(0, {tests!r})
from test_zz_no_alloc import _select, CALLS
torch.cuda.set_device(0)
rng = np.random.default_rng(7)
count, position, settings = CALLS[1]
logits = torch.from_numpy((rng.standard_normal(count) * 4).astype(np.float32)).cuda()
first = _select("select_static", logits, position, **settings)    # the device's first call: the set-up
second = _select("select_static", logits, position, **settings)
want = _select("select", logits, position, **settings)
for a, b in ((first, want), (second, want)):
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
print("fresh-process static selection ok")
"""


def test_first_call_in_a_fresh_process(cuda):
    code = FRESH.format(root=ROOT, tests=os.path.join(ROOT, "tests"))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "fresh-process static selection ok" in r.stdout
