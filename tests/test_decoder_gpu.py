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


def test_qwen3_0_6b_configs2_greedy_decode_token_for_token(cuda):
    """configs[2] exactly: Qwen3-0.6B (28 layers, hidden 1024, GQA 16/8 x 128,
    QK-norm, RoPE 1e6, SwiGLU 3072, tied 151,936 vocabulary: Q4_0 matmuls, a
    Q6_K table), a 512-token prompt of uniform random ids as one step, then
    256 greedy steps from the replayed graph: every token and the final
    logits bit for bit against the oracle."""
    run_both(M.qwen3_0_6b(context=4096), 512, 256, [512], seed=7)


def test_llama_3_2_1b_full_size_exact_path(cuda):
    """configs[3]'s architecture at full size on the exact path (16 layers,
    hidden 2048, 32/8 x 64, SwiGLU 8192, vocabulary 128,256, RoPE 5e5 with
    llama3 factors, a Q6_K output layer): a 512-token step, then 16 greedy
    steps, bit for bit against the oracle."""
    run_both(M.llama_3_2_1b(context=1024), 512, 16, [512], seed=11)


def test_gemma_3_1b_full_size_window_wraps(cuda):
    """configs[4]'s architecture at full size (26 layers, hidden 1152, 4/1 x
    256, window 512 on 5 of 6 layers, GeGLU-tanh 6912, post-norms, tied
    262,144 vocabulary): a 704-token prompt in steps of 128 (so a windowed
    layer's ring is 640 slots and wraps, and the window of 512 cuts keys
    off), then 16 greedy steps, bit for bit against the oracle."""
    run_both(M.gemma_3_1b(context=1024), 704, 16, [128] * 5 + [64], seed=13)
