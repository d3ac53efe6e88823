"""The tensor-core attention for prefill steps (cb_attention_run with
CB_RUN_TENSOR; the decoder's CB_DECODER_TENSOR_PREFILL): the attention of
attention.wgsl main :138-360 (causal, windowed, scale·log2e, softmax in log2
units) with queries and probabilities rounded to f16 and the sums made by
the tensor cores.

Parity tier: tolerance. Every output row of every head lies within
TOL·max(1, max|ref|) of an f64 softmax over the same f16 caches (the bound
the tensor-form products keep, 1e-3 of the largest value, doubled for the
two f16 roundings: q·scale and p); shapes the form does not take keep the
exact form's bits (the oracle's)."""
import math

import numpy as np
import pytest
import torch

import charlotte_b200 as cb
import oracle as O

pytestmark = pytest.mark.gpu

TOL = 2e-3


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def f16_cache(rng, slots, hkv, d, scale=1.0):
    return (rng.standard_normal((slots, hkv, d)) * scale).astype(np.float16).view(np.uint16)


def run(q, kc, vc, *, position, tokens, d, hq, hkv, slots, window, flags):
    max_chunks = (position + tokens + 63) // 64
    out = torch.zeros((tokens, hq * d), dtype=torch.float32, device="cuda")
    partials = torch.zeros(max_chunks * tokens * hq * d, dtype=torch.float32, device="cuda")
    stats = torch.zeros(max_chunks * tokens * hq * 2, dtype=torch.float32, device="cuda")
    tickets = torch.zeros(cb.lib().cb_attention_tickets(tokens, hq, hkv), dtype=torch.int32, device="cuda")
    cb.run("attention", query=q, key_cache=kc, value_cache=vc, out=out, partials=partials, stats=stats,
           tickets=tickets, position=0, position0=position, tokens=tokens, head_dim=d, query_heads=hq, kv_heads=hkv,
           slots=slots, window=window, max_chunks=max_chunks,
           scale_log2e=float(np.float32((1.0 / math.sqrt(d)) * 1.4426950408889634)), flags=flags)
    torch.cuda.synchronize()
    cb.check(cb.lib().cb_fault_check(None))
    return out


def softmax_f64(q, kc, vc, *, position, tokens, d, hq, hkv, slots, window):
    """[tokens, hq·d] f64 on the GPU: exp(s - max) over the row's live keys."""
    G = hq // hkv
    kf = kc.view(torch.float16).double().view(slots, hkv, d)
    vf = vc.view(torch.float16).double().view(slots, hkv, d)
    qf = q.double().view(tokens, hq, d)
    last = position + tokens - 1
    keys = torch.arange(0, last + 1, device="cuda")
    kk = kf[keys % slots]                       # [keys, hkv, d]
    vv = vf[keys % slots]
    out = torch.empty((tokens, hq, d), dtype=torch.float64, device="cuda")
    pos = position + torch.arange(tokens, device="cuda")
    early = torch.clamp(pos + 1 - window, min=0)
    live = (keys[None, :] <= pos[:, None]) & (keys[None, :] >= early[:, None])   # [tokens, keys]
    for h in range(hq):
        g = h // G
        s = qf[:, h] @ kk[:, g].T / math.sqrt(d)        # [tokens, keys]
        s = s.masked_fill(~live, -math.inf)
        w = torch.softmax(s, dim=1)
        out[:, h] = w @ vv[:, g]
    return out.view(tokens, hq * d)


CASES = [
    # d, Hq, Hkv, window, position, tokens
    (64, 32, 8, 1 << 30, 0, 512),       # Llama-3.2-1B's heads, a first prefill block
    (64, 32, 8, 1 << 30, 1536, 512),    # the last block of a 2,048-token prompt
    (128, 16, 8, 1 << 30, 0, 512),      # Qwen3-0.6B's heads
    (128, 16, 8, 1 << 30, 700, 130),    # ragged: a position inside a tile, rows past the last block
    (128, 8, 8, 1 << 30, 33, 100),      # one query head a kv head
    (64, 32, 4, 300, 900, 256),         # eight a kv head, a window shorter than the step's reach
    (128, 16, 8, 64, 0, 200),           # a window of one tile
    (64, 32, 8, 1 << 30, 5, 17),        # a short step
]


@pytest.mark.parametrize("case", CASES, ids=[f"d{c[0]}_{c[1]}x{c[2]}_w{min(c[3], 9999)}_p{c[4]}_t{c[5]}"
                                             for c in CASES])
def test_tensor_attention_within_tolerance(cuda, case):
    d, hq, hkv, window, position, tokens = case
    rng = np.random.default_rng(d + hq + position + tokens)
    slots = 4096
    kc = dev(f16_cache(rng, slots, hkv, d, 2.0))
    vc = dev(f16_cache(rng, slots, hkv, d))
    q = dev(rng.standard_normal((tokens, hq * d)).astype(np.float32))
    shape = dict(position=position, tokens=tokens, d=d, hq=hq, hkv=hkv, slots=slots, window=window)
    got = run(q, kc, vc, flags=cb.RUN_TENSOR, **shape).double()
    ref = softmax_f64(q, kc, vc, **shape)
    err = (got - ref).abs().view(tokens, hq, d).amax(dim=2)
    bound = TOL * torch.clamp(ref.abs().view(tokens, hq, d).amax(dim=2), min=1.0)
    worst = float((err / bound).max())
    assert worst <= 1.0, f"worst row-head error {worst:.2f} of the bound"
    # and it is a different computation from the exact form (the flag took effect)
    exact = run(q, kc, vc, flags=0, **shape)
    assert not torch.equal(exact.double(), got)


@pytest.mark.parametrize("d,hq,hkv,tokens", [(256, 4, 1, 64), (128, 16, 8, 1), (128, 12, 4, 64)])
def test_shapes_outside_the_tensor_form_stay_exact(cuda, d, hq, hkv, tokens):
    """Head dimension 256, a one-row step (under 16 positions) and three
    query heads a kv head take the exact form under the flag: the oracle's
    bits."""
    rng = np.random.default_rng(d + hq + tokens)
    slots, position = 1024, 300
    kc = f16_cache(rng, slots, hkv, d, 2.0)
    vc = f16_cache(rng, slots, hkv, d)
    q = rng.standard_normal((tokens, hq * d)).astype(np.float32)
    scale = float(np.float32((1.0 / math.sqrt(d)) * 1.4426950408889634))
    got = run(dev(q), dev(kc), dev(vc), position=position, tokens=tokens, d=d, hq=hq, hkv=hkv, slots=slots,
              window=1 << 30, flags=cb.RUN_TENSOR).cpu().numpy()
    for t in (0, tokens - 1):
        want = O.attention_row(q[t], position + t, kc, vc, slots, 1 << 30, scale, d, hq, hkv)
        np.testing.assert_array_equal(got[t], want)
