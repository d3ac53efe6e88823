"""The tensor-core form of the matrix products (CB_MATMUL_TENSOR: tcgen05
MMA, f16 operands, f32 accumulation in tensor memory) against f64 products
over the reference's own dequantized weights.

Parity tier: tolerance, as BASELINE states it for GEMV/GEMM outputs and
logits: max |y - y_f64| <= 1e-3 * max |y_f64| (TOL below). The weights are
decoded exactly first (the same decode the exact forms use), then rounded to
f16 with x. Cases cover each format, each epilogue, ragged token and row
tails (partial 128-token and 128-slot tiles), a K that ends in half a
64-wide block, and a step long enough to cycle the 4-stage ring many times."""
import numpy as np
import pytest
import torch

import charlotte_b200 as cb
import oracle as O
from charlotte_b200 import synth

pytestmark = pytest.mark.gpu

TOL = 1e-3


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def weight(rng, fmt, rows, K):
    nb = rows * K // O.BLOCK_WEIGHTS[fmt]
    stored = synth.blocks(rng, fmt, rows, K)
    return stored, synth.to_piece(fmt, stored), nb


def exact(fmt, stored, rows, K, x):
    W = O.dequant_stored(fmt, stored).reshape(rows, K).astype(np.float64)
    return x.astype(np.float64) @ W.T


def run(fmt, K, members, x, outs, **kw):
    cb.matmul(fmt, K, members, x, outs, flags=cb.MATMUL_TENSOR, **kw)
    torch.cuda.synchronize()
    cb.check(cb.lib().cb_fault_check(None))


def within(got, want):
    err = np.max(np.abs(got.astype(np.float64) - want))
    scale = np.max(np.abs(want))
    assert err <= TOL * scale, f"max err {err:.3e} = {err / scale:.2e} of max|y| {scale:.3e}"
    return err / scale


CASES = [
    (O.Q4_0, 4096, 1024, 512),
    (O.Q4_0, 1024, 3072, 200),   # ragged token tile
    (O.Q4_0, 300, 1152, 130),    # ragged slot tile, 18 K blocks
    (O.Q4_0, 128, 96, 128),      # K ends in half a block
    (O.Q8_0, 1024, 2048, 384),
    (O.Q6_K, 2048, 1024, 256),
    (O.Q6_K, 1000, 2048, 1),
    (O.Q4_1, 1024, 3072, 256),
    (O.BF16, 1024, 1024, 128),
]


@pytest.mark.parametrize("fmt,rows,K,tokens", CASES)
def test_tensor_write_within_tolerance(cuda, fmt, rows, K, tokens):
    rng = np.random.default_rng(rows + K * 3 + tokens + fmt)
    stored, piece, nb = weight(rng, fmt, rows, K)
    x = synth.activations(rng, tokens, K)
    y = torch.full((tokens, rows), float("nan"), dtype=torch.float32, device="cuda")
    run(fmt, K, [(dev(piece), nb, 0, rows, 0)], dev(x), [y])
    within(y.cpu().numpy(), exact(fmt, stored, rows, K, x))


def test_tensor_qkv(cuda):
    rng = np.random.default_rng(41)
    K, T = 1024, 300
    x = synth.activations(rng, T, K)
    members, wants, outs = [], [], []
    for rows in (2048, 1000, 1000):
        stored, piece, nb = weight(rng, O.Q4_0, rows, K)
        members.append((dev(piece), nb, 0, rows, 0))
        wants.append(exact(O.Q4_0, stored, rows, K, x))
        outs.append(torch.zeros((T, rows), dtype=torch.float32, device="cuda"))
    run(O.Q4_0, K, members, dev(x), outs, epilogue=cb.QKV)
    for o, w in zip(outs, wants):
        within(o.cpu().numpy(), w)


@pytest.mark.parametrize("activation", [cb.SILU, cb.GELU_TANH])
def test_tensor_gated(cuda, activation):
    rng = np.random.default_rng(43 + activation)
    F, K, T = 3000, 1024, 257
    gs, gp, gnb = weight(rng, O.Q4_0, F, K)
    us, up, unb = weight(rng, O.Q4_0, F, K)
    x = synth.activations(rng, T, K)
    y = torch.zeros((T, F), dtype=torch.float32, device="cuda")
    run(O.Q4_0, K, [(dev(gp), gnb, 0, F, 0), (dev(up), unb, 0, F, 0)], dev(x), [y], epilogue=cb.GATED,
        activation=activation)
    g = exact(O.Q4_0, gs, F, K, x)
    u = exact(O.Q4_0, us, F, K, x)
    if activation == cb.SILU:
        act = g / (1.0 + np.exp(-g))
    else:
        act = 0.5 * g * (1.0 + np.tanh(0.7978845608028654 * (g + 0.044715 * g ** 3)))
    within(y.cpu().numpy(), act * u)


def test_tensor_gated_by_input(cuda):
    rng = np.random.default_rng(47)
    rows, K, T = 640, 1024, 150
    stored, piece, nb = weight(rng, O.Q4_0, rows, K)
    x = synth.activations(rng, T, K)
    u = rng.standard_normal((T + 3, 1000)).astype(np.float32)
    y = torch.zeros((T, rows), dtype=torch.float32, device="cuda")
    run(O.Q4_0, K, [(dev(piece), nb, 0, rows, 0)], dev(x), [y], epilogue=cb.GATED_BY_INPUT,
        activation=cb.SILU, gate_input=dev(u), gate_input_stride=1000, gate_input_column=100,
        gate_input_token=2)
    t = exact(O.Q4_0, stored, rows, K, x)
    within(y.cpu().numpy(), t / (1.0 + np.exp(-t)) * u[2:2 + T, 100:100 + rows])
