"""Failure detection without a GPU fault: every wait of a kernel on a copy is
bounded, and one that runs out sets the device's fault word, drains the
CTA's copies and returns; the host reads the word (cb_fault_check) and
reports a failed step (CB_ERROR_STEP), and the context stays usable.

The waits are made to run out on purpose with cb_debug_spin_limit(0): the
first wait on each copy then gives up at once, without polling, before a
copy from HBM can land. Nothing faults, traps or hangs; the copies are real and
land (the drain takes the full bound). Afterwards the limit is restored and
the same work gives the oracle's bits again."""
import numpy as np
import pytest
import torch

import charlotte_b200 as cb
import oracle as O
from charlotte_b200 import model as M
from charlotte_b200 import synth

pytestmark = pytest.mark.gpu


@pytest.fixture
def short_waits():
    yield lambda polls: cb.check(cb.lib().cb_debug_spin_limit(polls))
    cb.lib().cb_debug_spin_limit(-1)


def test_product_whose_wait_runs_out_reports_a_failed_step(cuda, short_waits):
    rng = np.random.default_rng(5)
    rows, K = 16384, 4096            # 37.7 MB of Q4_0: many batches a warp, streamed
    stored = synth.blocks(rng, O.Q4_0, rows, K)
    piece_h = synth.to_piece(O.Q4_0, stored)
    nb = rows * K // 32
    piece = torch.from_numpy(piece_h).cuda()
    xh = synth.activations(rng, 1, K)
    x = torch.from_numpy(xh).cuda()
    y = torch.zeros((1, rows), dtype=torch.float32, device="cuda")
    assert cb.lib().cb_fault_check(None) == cb.OK
    short_waits(0)
    cb.matmul(O.Q4_0, K, [(piece, nb, 0, rows, 0)], x, [y])
    torch.cuda.synchronize()
    import ctypes
    bits = ctypes.c_uint(0)
    assert cb.lib().cb_fault_check(ctypes.byref(bits)) == cb.ERROR_STEP
    assert bits.value & 1, bits.value
    assert "bounded wait" in cb.last_error()
    # the word was cleared by the read; the full bound again gives the bits
    short_waits(-1)
    cb.matmul(O.Q4_0, K, [(piece, nb, 0, rows, 0)], x, [y])
    torch.cuda.synchronize()
    assert cb.lib().cb_fault_check(None) == cb.OK
    np.testing.assert_array_equal(y.cpu().numpy(), O.matmul(O.Q4_0, piece_h, nb, rows, K, xh))


def test_decoder_step_after_a_timed_out_step_gives_the_oracle_bits(cuda, short_waits):
    """A Qwen3-0.6B decoder: a one-token step whose waits run out (its 127 MB
    head streams from HBM) fails with CB_ERROR_STEP; the decoder clears its
    ticket words; the same step run again, and a decode step after it, equal
    the oracle's records and logits bit for bit."""
    from oracle.model import OracleDecoder
    m = M.synthesize(M.qwen3_0_6b(context=256), seed=31)
    rng = np.random.default_rng(6)
    prompt = rng.integers(0, m.arch.vocab, 12).astype(np.uint32)
    dec = M.Decoder(m, max_step_tokens=16)
    dec.prefill(prompt[:11])
    short_waits(0)
    with pytest.raises(cb.CharlotteError) as e:
        dec.step(prompt[11:12], 11)
    assert e.value.status == cb.ERROR_STEP
    short_waits(-1)
    rec = dec.step(prompt[11:12], 11)
    got = dec.logits()
    toks, failed = dec.generate(2)
    assert not failed.any()
    od = OracleDecoder(m)
    orec, olg = od.step(prompt, 0)
    np.testing.assert_array_equal(rec, orec)
    np.testing.assert_array_equal(got, olg)
    want = []
    prev = orec[0]
    for i in range(2):
        r, _ = od.step([prev], 12 + i)
        want.append(int(r[0]))
        prev = r[0]
    assert toks.tolist() == want
    dec.close()
    od.close()
