"""The oracle's pins (tests/test_oracle_pins.py: every dequantizer, the Q6_K
repack, the f16 conversions, Philox, the rope turns and the draw against the
reference's own CPU code in oracle/_ref) run again on the GPU box, where the
GPU tests run, so a record of that run shows the oracle pinned there too;
and the GPU's own draw (cb_select_merge_run over one candidate list) against
the reference's f64 draw given the same uniform."""
import ctypes
import math
import os
import subprocess
import sys

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_oracle_pins_pass_here_with_nothing_skipped(cuda):
    assert O.ref() is not None, "oracle/_ref is missing: the pins cannot run"
    r = subprocess.run([sys.executable, "-m", "pytest", os.path.join(ROOT, "tests", "test_oracle_pins.py"), "-q",
                        "-m", "not gpu", "-p", "no:cacheprovider", "-rs"], capture_output=True, text=True,
                       cwd=ROOT, timeout=900)
    tail = r.stdout[-2000:]
    assert r.returncode == 0, tail
    assert " passed" in tail and "skipped" not in tail, tail


def test_gpu_draw_equals_the_reference_f64_draw(cuda):
    """The draw kernel over the reference draw test's candidates, five
    settings x 100 positions: the token is the reference's f64 choice for the
    kernel's own uniform (which equals the reference's Philox uniform),
    except within f32 rounding of a decision (margin < 1e-5, at most 1%)."""
    import torch
    import charlotte_b200 as cb
    from test_oracle_pins import DRAW_SETTINGS, _candidates, _pairs, _ref_draw, _ref_uniform
    logits, tokens = _candidates(2)
    lists = torch.from_numpy(_pairs(logits, tokens).view(np.int32)).cuda()
    cand = torch.zeros(128, dtype=torch.int32, device="cuda")
    rec = torch.zeros(4, dtype=torch.int32, device="cuda")
    compared = near = 0
    for s in DRAW_SETTINGS:
        for position in range(100):
            cb.run("select_merge", lists_data=lists, lists=1, rows=1, candidates=cand, sampled=rec, position=0,
                   position0=position, tokens=1, seed0=42, seed1=0, top_k=s[1], temperature=s[0], top_p=s[2],
                   min_p=s[3], log_min_p=math.log(s[3]) if s[3] > 0 else 0.0)
            got = rec.cpu().numpy().view(np.uint32)
            assert got[1] == 0
            assert got[2] == _ref_uniform(42, position + 1).view(np.uint32)
            chosen, margin = _ref_draw(logits, tokens, s, float(got[2:3].view(np.float32)[0]))
            if margin < 1e-5:
                near += 1
                continue
            compared += 1
            assert got[0] == tokens[chosen], (s, position)
    cb.check(cb.lib().cb_fault_check(None))
    assert near * 100 <= compared
