"""The streamed multi-token form of the matrix products (steps of 2 to 64
tokens: each weight decoded once and applied to up to 16 tokens) against the
CPU oracle, bit for bit, and against the tiled form: both exact forms must
give the same bits for the same step (matmul.h 'Determinism')."""
import numpy as np
import pytest
import torch

import charlotte_b200 as cb
import oracle as O
from charlotte_b200 import synth

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def weight(rng, fmt, rows, K):
    nb = rows * K // O.BLOCK_WEIGHTS[fmt]
    stored = synth.blocks(rng, fmt, rows, K)
    return stored, synth.to_piece(fmt, stored), nb


def run(fmt, K, members, x, outs, **kw):
    cb.matmul(fmt, K, members, x, outs, **kw)
    torch.cuda.synchronize()
    cb.check(cb.lib().cb_fault_check(None))


def assert_exact(got, want):
    got = np.asarray(got, np.float32).reshape(-1)
    want = np.asarray(want, np.float32).reshape(-1)
    bad = np.flatnonzero(got != want)
    assert bad.size == 0, f"{bad.size} of {got.size} outputs differ; first at {bad[:5]}: {got[bad[:5]]} vs {want[bad[:5]]}"


def act_of(activation, v):
    return np.vectorize(lambda g: O.lib().or_activate(activation, float(g)), otypes=[np.float32])(v)


CASES = [
    (O.Q4_0, 4096, 1024, 2),
    (O.Q4_0, 1024, 3072, 5),     # 8 tokens a pass, 3 live
    (O.Q4_0, 1023, 2048, 16),    # an odd row count: the last pair half live
    (O.Q4_0, 77, 64, 3),         # 2 groups: 30 ranges empty
    (O.Q8_0, 1152, 6912, 9),     # Gemma down width, 16 a pass (x of 9 tokens staged)
    (O.Q8_0, 333, 1024, 40),     # several token groups
    (O.Q6_K, 4096, 1024, 7),
    (O.Q6_K, 300, 2048, 64),
    (O.Q4_1, 1024, 3072, 5),
    (O.BF16, 333, 1024, 40),
    # two row pairs a batch (large products), the last batch one row live
    (O.Q4_0, 4097, 1024, 3),
    (O.Q8_0, 2049, 1152, 8),
    (O.Q6_K, 65537, 256, 2),
]


@pytest.mark.parametrize("fmt,rows,K,tokens", CASES)
def test_streamed_write_bit_exact(cuda, fmt, rows, K, tokens):
    rng = np.random.default_rng(rows * 5 + K + tokens + fmt)
    stored, piece, nb = weight(rng, fmt, rows, K)
    x = synth.activations(rng, tokens, K)
    y = torch.full((tokens, rows), float("nan"), dtype=torch.float32, device="cuda")
    run(fmt, K, [(dev(piece), nb, 0, rows, 0)], dev(x), [y], flags=cb.MATMUL_STREAMED)
    assert_exact(y.cpu().numpy(), O.matmul(fmt, piece, nb, rows, K, x))


@pytest.mark.parametrize("tokens", [2, 12, 33])
def test_streamed_and_tiled_forms_agree(cuda, tokens):
    rng = np.random.default_rng(tokens)
    rows, K = 2000, 2048
    stored, piece, nb = weight(rng, O.Q4_0, rows, K)
    x = dev(synth.activations(rng, tokens, K))
    p = dev(piece)
    ys = torch.zeros((tokens, rows), dtype=torch.float32, device="cuda")
    yt = torch.zeros((tokens, rows), dtype=torch.float32, device="cuda")
    run(O.Q4_0, K, [(p, nb, 0, rows, 0)], x, [ys], flags=cb.MATMUL_STREAMED)
    run(O.Q4_0, K, [(p, nb, 0, rows, 0)], x, [yt], flags=cb.MATMUL_TILED)
    assert_exact(ys.cpu().numpy(), yt.cpu().numpy())


def test_streamed_qkv(cuda):
    rng = np.random.default_rng(6)
    K, T = 1024, 6
    x = synth.activations(rng, T, K)
    members, wants, outs = [], [], []
    for rows in (2048, 1023, 1025):
        stored, piece, nb = weight(rng, O.Q4_0, rows, K)
        members.append((dev(piece), nb, 0, rows, 0))
        wants.append(O.matmul(O.Q4_0, piece, nb, rows, K, x))
        outs.append(torch.zeros((T, rows), dtype=torch.float32, device="cuda"))
    run(O.Q4_0, K, members, dev(x), outs, epilogue=cb.QKV, flags=cb.MATMUL_STREAMED)
    for o, w in zip(outs, wants):
        assert_exact(o.cpu().numpy(), w)


@pytest.mark.parametrize("activation", [cb.SILU, cb.GELU_TANH])
@pytest.mark.parametrize("T,F", [(3, 3072), (7, 3072), (8, 2049), (16, 3072), (21, 3072)])
def test_streamed_gated(cuda, activation, T, F):
    """T = 7, 8 at 2,048+ slots: batches of two outputs' gate rows then their up
    rows (F = 2,049: the last batch one output live)."""
    rng = np.random.default_rng(T + activation)
    K = 1024
    gs, gp, gnb = weight(rng, O.Q4_0, F, K)
    us, up, unb = weight(rng, O.Q4_0, F, K)
    x = synth.activations(rng, T, K) * 4
    y = torch.zeros((T, F), dtype=torch.float32, device="cuda")
    run(O.Q4_0, K, [(dev(gp), gnb, 0, F, 0), (dev(up), unb, 0, F, 0)], dev(x), [y], epilogue=cb.GATED,
        activation=activation, flags=cb.MATMUL_STREAMED)
    gate = O.matmul(O.Q4_0, gp, gnb, F, K, x)
    upv = O.matmul(O.Q4_0, up, unb, F, K, x)
    assert_exact(y.cpu().numpy(), (act_of(activation, gate) * upv).astype(np.float32))


def test_streamed_gated_by_input(cuda):
    rng = np.random.default_rng(18)
    rows, K, T = 640, 1024, 5
    stored, piece, nb = weight(rng, O.Q4_0, rows, K)
    x = synth.activations(rng, T, K)
    u = rng.standard_normal((T + 3, 1000)).astype(np.float32)
    y = torch.zeros((T, rows), dtype=torch.float32, device="cuda")
    run(O.Q4_0, K, [(dev(piece), nb, 0, rows, 0)], dev(x), [y], epilogue=cb.GATED_BY_INPUT,
        activation=cb.GELU_TANH, gate_input=dev(u), gate_input_stride=1000, gate_input_column=100,
        gate_input_token=2, flags=cb.MATMUL_STREAMED)
    t = O.matmul(O.Q4_0, piece, nb, rows, K, x)
    assert_exact(y.cpu().numpy(), act_of(cb.GELU_TANH, t) * u[2:2 + T, 100:100 + rows])
