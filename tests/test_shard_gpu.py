"""The vocabulary-split head (charlotte_b200.shard) on one GPU, its ranks
emulated in turn: every rank's shard of the head, its candidates with global
ids (cb_select_run, candidates_only), the lists stacked as an all-gather
leaves them, and the merge and draw (cb_select_merge_run). Parity tier:
bit-exact — the merged candidates equal one selection's over the whole
vocabulary, and the greedy tokens of several fed steps equal the batched
decoder's own (whole-head) steps."""
import numpy as np
import pytest
import torch

import charlotte_b200 as cb
from charlotte_b200 import model as M
from charlotte_b200 import shard

pytestmark = pytest.mark.gpu


def emulated_step(heads, position, ids=None):
    """One batched step with `len(heads)` emulated ranks sharing one decoder."""
    heads[0].body(position, ids)
    for h in heads:
        with torch.cuda.stream(h.stream):
            h.normed_all.copy_(h.local_normed())
        h.shard_candidates()
    with torch.cuda.stream(heads[0].stream):
        stacked = torch.stack([h.cand for h in heads])
        for h in heads:
            h.cand_all.copy_(stacked)
    heads[0].merge(position)
    torch.cuda.synchronize()
    return heads[0].sampled_all.cpu().numpy().view(np.uint32), heads[0].merged.cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("world", [2, 3, 8])
def test_split_head_equals_whole_head(cuda, world):
    arch = M.tiny("gemma3")
    m = M.synthesize(arch, seed=31)
    rng = np.random.default_rng(7)
    S, P, steps = 4, 24, 6
    prompts = [rng.integers(0, arch.vocab, P).astype(np.uint32) for _ in range(S)]
    nxt = rng.integers(0, arch.vocab, S).astype(np.uint32)

    ref = M.BatchDecoder(m, S, max_step_tokens=32)
    for s, p in enumerate(prompts):
        ref.prefill_sequence(s, p)
    want_first = ref.step_batch(nxt, P)
    want_logits = [ref.logits_row(s) for s in range(S)]
    want_toks, _ = ref.generate(steps)
    ref.close()

    dec = M.BatchDecoder(m, S, max_step_tokens=32)
    for s, p in enumerate(prompts):
        dec.prefill_sequence(s, p)
    heads = [shard.SplitHead(dec, S, world, r) for r in range(world)]
    got, merged = emulated_step(heads, P, nxt)
    np.testing.assert_array_equal(got[:, 0], want_first[:, 0])
    # the merged candidates are the whole vocabulary's top 64
    for s in range(S):
        lg = torch.from_numpy(want_logits[s]).cuda()
        parts = torch.empty(cb.lib().cb_select_tiles(arch.vocab) * 128, dtype=torch.int32, device="cuda")
        ticket = torch.zeros(cb.lib().cb_select_tickets(arch.vocab), dtype=torch.int32, device="cuda")
        cand = torch.empty(128, dtype=torch.int32, device="cuda")
        samp = torch.empty(4, dtype=torch.int32, device="cuda")
        cb.run("select", logits=lg, count=arch.vocab, partials=parts, ticket=ticket, candidates=cand, sampled=samp,
               top_k=1)
        np.testing.assert_array_equal(merged[s], cand.cpu().numpy().view(np.uint32))
    toks = []
    for i in range(steps):
        got, _ = emulated_step(heads, P + 1 + i)
        toks.append(got[:, 0].copy())
    dec.close()
    np.testing.assert_array_equal(np.array(toks), want_toks)
