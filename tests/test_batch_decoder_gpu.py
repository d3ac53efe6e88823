"""Batched decode (cb_decoder_create_batch): several independent sequences
stepping together, one token each at a common position, through the same C
ABI. Parity tier: bit-exact — every sequence's greedy tokens and logits equal
those of the same sequence decoded alone by a one-sequence decoder (which is
itself bit-exact with the oracle), for each model family, including Gemma's
sliding-window rings wrapping, and with the batch fed from host ids
(cb_decoder_step_batch) or from each row's last draw (the replayed graph)."""
import numpy as np
import pytest

import charlotte_b200  # noqa: F401
from charlotte_b200 import model as M

pytestmark = pytest.mark.gpu


def alone(m, prompt, steps):
    dec = M.Decoder(m, max_step_tokens=64)
    rec = dec.prefill(prompt)
    first = dec.logits()
    toks, failed = dec.generate(steps)
    last = dec.logits()
    dec.close()
    return int(rec[0]), first, toks, last


@pytest.mark.parametrize("kind", ["qwen3", "llama", "gemma3"])
def test_batch_matches_sequences_alone(cuda, kind):
    arch = M.tiny(kind)
    m = M.synthesize(arch, seed=21)
    rng = np.random.default_rng(3)
    S, P, steps = 5, 40, 24   # gemma's window of 16 wraps its rings
    prompts = [rng.integers(0, arch.vocab, P).astype(np.uint32) for _ in range(S)]
    bd = M.BatchDecoder(m, S, max_step_tokens=64)
    firsts = []
    for s, p in enumerate(prompts):
        rec = bd.prefill_sequence(s, p)
        firsts.append(int(rec[0]))
    first_logits = [bd.logits_row(s) for s in range(S)]
    toks, failed = bd.generate(steps)
    assert not failed.any()
    last_logits = [bd.logits_row(s) for s in range(S)]
    bd.close()
    for s, p in enumerate(prompts):
        tok0, l0, want, lw = alone(m, p, steps)
        assert firsts[s] == tok0
        np.testing.assert_array_equal(first_logits[s], l0)
        assert toks[:, s].tolist() == want.tolist(), (s, toks[:, s].tolist(), want.tolist())
        np.testing.assert_array_equal(last_logits[s], lw)


def test_batch_step_from_host_ids(cuda):
    """A batched step fed from host ids gives each row the bits of a
    one-token step of its sequence alone."""
    arch = M.tiny("qwen3")
    m = M.synthesize(arch, seed=8)
    rng = np.random.default_rng(4)
    S, P = 7, 20
    prompts = [rng.integers(0, arch.vocab, P).astype(np.uint32) for _ in range(S)]
    nxt = rng.integers(0, arch.vocab, S).astype(np.uint32)
    bd = M.BatchDecoder(m, S, max_step_tokens=32)
    for s, p in enumerate(prompts):
        bd.prefill_sequence(s, p)
    recs = bd.step_batch(nxt, P)
    rows = [bd.logits_row(s) for s in range(S)]
    bd.close()
    for s, p in enumerate(prompts):
        dec = M.Decoder(m, max_step_tokens=32)
        dec.prefill(p)
        rec = dec.step(nxt[s:s + 1], P)
        np.testing.assert_array_equal(rows[s], dec.logits())
        assert int(recs[s, 0]) == int(rec[0])
        dec.close()


@pytest.mark.parametrize("S,rows", [(64, (0, 21, 42, 63)), (8, (0, 3, 7))])
def test_gemma_3_1b_batch_rows_match_sequences_alone(cuda, S, rows):
    """configs[4]'s shape at full size: 64 sequences batched (each with its
    own caches, a windowed layer's ring of 512 + 64 slots wrapping over the
    620 positions), 8 batched greedy steps; the given rows give the tokens
    and logits of their sequences decoded alone (themselves bit-exact with
    the oracle at full size). 8 sequences (one GPU's share at N = 8) take the
    streamed products with two row pairs a batch and the windowed layers'
    attention over clusters of 9 chunk CTAs."""
    m = M.synthesize(M.gemma_3_1b(context=1024), seed=23)
    rng = np.random.default_rng(9)
    P, steps = 612, 8
    prompts = [rng.integers(0, m.arch.vocab, P).astype(np.uint32) for _ in range(S)]
    bd = M.BatchDecoder(m, S, max_step_tokens=64)
    firsts = [int(bd.prefill_sequence(s, p)[0]) for s, p in enumerate(prompts)]
    toks, failed = bd.generate(steps)
    assert not failed.any()
    last = {r: bd.logits_row(r) for r in rows}
    bd.close()
    for r in rows:
        dec = M.Decoder(m, max_step_tokens=64)
        rec = dec.prefill(prompts[r])
        assert firsts[r] == int(rec[0])
        want, wf = dec.generate(steps)
        assert not wf.any()
        assert toks[:, r].tolist() == want.tolist(), r
        np.testing.assert_array_equal(last[r], dec.logits())
        dec.close()
