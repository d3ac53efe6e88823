"""The whole decoder through the C ABI (cb_decoder_*) against the oracle's
pass over the same seeded weights. Parity tier (BASELINE): greedy token
sequences identical, token for token; logits bit-exact (zeros by value),
which is stronger than the stated tolerance 1e-3·max|logit|, also checked.

Prompts are stepped unevenly on the GPU (the reference's batch invariance:
a token's bits do not depend on its step) while the oracle steps every token
alone; decode runs as the replayed CUDA graph, fed on the device."""
import numpy as np
import pytest

import charlotte_b200  # noqa: F401
from charlotte_b200 import model as M
from oracle.model import OracleDecoder

pytestmark = pytest.mark.gpu


def run_both(arch, prompt_len, steps, split, seed=0):
    m = M.synthesize(arch, seed=seed)
    rng = np.random.default_rng(seed + 100)
    prompt = rng.integers(0, arch.vocab, prompt_len).astype(np.uint32)
    dec = M.Decoder(m, max_step_tokens=max(split))
    od = OracleDecoder(m)
    # GPU: the prompt in uneven steps, the last one drawing
    at = 0
    rec = None
    for i, n in enumerate(split):
        part = prompt[at: at + n]
        rec = dec.step(part, at, logits=(at + n == prompt_len))
        at += n
    assert at == prompt_len
    gpu_logits = dec.logits()
    orec, olg = od.step(prompt, 0)
    np.testing.assert_array_equal(gpu_logits, olg)
    assert np.max(np.abs(gpu_logits - olg)) <= 1e-3 * np.max(np.abs(olg))
    np.testing.assert_array_equal(rec, orec)
    toks, failed = dec.generate(steps)
    assert not failed.any()
    want = []
    prev = orec[0]
    for i in range(steps):
        r, lg = od.step([prev], prompt_len + i)
        want.append(int(r[0]))
        prev = r[0]
    assert toks.tolist() == want, (toks.tolist(), want)
    np.testing.assert_array_equal(dec.logits(), lg)
    dec.close()
    od.close()
    return toks


@pytest.mark.parametrize("kind", ["qwen3", "llama", "gemma3"])
def test_tiny_decoder_matches_oracle(cuda, kind):
    run_both(M.tiny(kind), 40, 12, [7, 33 - 7, 7], seed=hash(kind) % 1000)


@pytest.mark.parametrize("matmul,down", [(2, 3), (30, 30)], ids=["q4_1_down", "bf16"])
def test_decoder_with_q4_1_and_bf16_weights(cuda, matmul, down):
    """Q4_1 down projections (as the real Qwen3 Q4_0 file has) and BF16
    layer weights through the whole decoder, token for token and logits bit
    for bit against the oracle."""
    import dataclasses
    arch = dataclasses.replace(M.tiny("qwen3"), matmul_format=matmul, down_format=down)
    run_both(arch, 24, 8, [5, 19], seed=11)


def test_gemma_window_ring_wraps(cuda):
    """A sliding-window layer's ring (window 16 + step slots) wraps several
    times over a 120-token prompt and 20 decode steps."""
    run_both(M.tiny("gemma3", context=256), 120, 20, [24] * 5, seed=5)


def test_qwen3_0_6b_greedy_decode_token_for_token(cuda):
    """configs[2]'s architecture at full size (28 layers, 151,936 vocab),
    a shorter run: 64-token prompt in two steps, 16 greedy steps."""
    run_both(M.qwen3_0_6b(), 64, 16, [40, 24], seed=7)


@pytest.mark.parametrize("kind", ["qwen3", "llama", "gemma3"])
def test_fused_step_matches_separate_launches(cuda, kind):
    """The fused one-token step (CB_DECODER_FUSED: one persistent launch,
    grid-wide barriers) gives the same tokens and logits, bit for bit, as the
    separate launches, fed from the device and from host ids."""
    arch = M.tiny(kind)
    m = M.synthesize(arch, seed=17)
    rng = np.random.default_rng(2)
    prompt = rng.integers(0, arch.vocab, 30).astype(np.uint32)
    out = {}
    for fused in (True, False):
        dec = M.Decoder(m, max_step_tokens=32, fused=fused)
        dec.prefill(prompt)
        toks, failed = dec.generate(20)
        assert not failed.any()
        lg = dec.logits()
        rec = dec.step(np.array([7], np.uint32), 50)
        out[fused] = (toks, lg, rec, dec.logits())
        dec.close()
    np.testing.assert_array_equal(out[True][0], out[False][0])
    np.testing.assert_array_equal(out[True][1], out[False][1])
    np.testing.assert_array_equal(out[True][2], out[False][2])
    np.testing.assert_array_equal(out[True][3], out[False][3])
