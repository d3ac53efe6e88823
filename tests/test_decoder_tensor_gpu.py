"""The decoder with CB_DECODER_TENSOR_PREFILL: prompt steps of 128 tokens or
more run their products on the tensor cores (f16 operands, f32
accumulation), decode steps stay exact.

Parity tier: tolerance (BASELINE: logits within 1e-3·max|logit|) against
the oracle's pass over the same seeded weights for the tiny models; at full
size (Llama-3.2-1B shapes, a 2,048-token prompt as four 512-token steps, the
configs[3] workload) against the exact GPU path, which is itself bit-exact
with the oracle on the tiny models. The worst relative error is recorded."""
import numpy as np
import pytest

import charlotte_b200  # noqa: F401
from charlotte_b200 import model as M
from oracle.model import OracleDecoder

pytestmark = pytest.mark.gpu

TOL = 1e-3


def rel_err(got, want):
    return float(np.max(np.abs(got.astype(np.float64) - want)) / np.max(np.abs(want)))


@pytest.mark.parametrize("kind", ["qwen3", "llama", "gemma3"])
def test_tiny_tensor_prefill_logits_within_tolerance(cuda, kind):
    arch = M.tiny(kind)
    m = M.synthesize(arch, seed=11)
    rng = np.random.default_rng(5)
    prompt = rng.integers(0, arch.vocab, 160).astype(np.uint32)
    dec = M.Decoder(m, max_step_tokens=160, tensor_prefill=True)
    dec.step(prompt, 0, logits=True)
    got = dec.logits()
    toks, failed = dec.generate(4)   # decode continues (exact form) after a tensor prefill
    assert not failed.any()
    dec.close()
    od = OracleDecoder(m)
    _, want = od.step(prompt, 0)
    od.close()
    e = rel_err(got, want)
    assert e <= TOL, f"{kind}: logits differ by {e:.2e} of max|logit|"


def test_llama_2048_prefill_tensor_vs_exact(cuda):
    """configs[3] at full size: a 2,048-token prompt as four 512-token steps,
    tensor form against the exact form on the GPU."""
    arch = M.llama_3_2_1b(context=2304)
    m = M.synthesize(arch, seed=4)
    rng = np.random.default_rng(9)
    prompt = rng.integers(0, arch.vocab, 2048).astype(np.uint32)
    out = {}
    for tensor in (False, True):
        dec = M.Decoder(m, max_step_tokens=512, tensor_prefill=tensor)
        for i in range(4):
            dec.step(prompt[512 * i: 512 * (i + 1)], 512 * i, logits=(i == 3))
        out[tensor] = dec.logits()
        dec.close()
    e = rel_err(out[True], out[False].astype(np.float64))
    assert e <= TOL, f"logits differ by {e:.2e} of max|logit|"
