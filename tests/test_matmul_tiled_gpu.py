"""The tiled (prefill) form of the matrix products against the CPU oracle.

Parity tier: bit-exact. Long steps take the tiled kernel by default, and any
step with CB_MATMUL_TILED, which these tests set. Every output must equal the
oracle's — the reference's prefill order, which is its decode order (matmul.wgsl tile_range :410, matmul.h
34-50) — bit for bit, and a token's outputs must be the bits the decode form
gives it alone. Shapes cover each tile shape the dispatch picks (long and
short steps, wide and narrow products), ragged token and row tails, ranges of
one group, several, unequal and mostly empty, and every epilogue."""
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
    kw.setdefault("flags", cb.MATMUL_TILED)
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
    # fmt, rows, K, tokens
    (O.Q4_0, 4096, 1024, 512),   # Qwen3 QKV at a 512-token step: the 128x128 tile
    (O.Q4_0, 1024, 2048, 512),   # Qwen3 O: few column tiles
    (O.Q4_0, 1024, 3072, 130),   # down, 3 groups a range, a ragged token tail
    (O.Q4_0, 300, 1152, 77),     # Gemma width: unequal ranges
    (O.Q4_0, 77, 64, 9),         # 2 groups: 30 ranges empty
    (O.Q4_0, 2048, 1024, 8),     # the shortest tiled step
    (O.Q8_0, 1024, 1024, 200),
    (O.Q8_0, 333, 6912, 33),
    (O.Q6_K, 4096, 1024, 64),
    (O.Q6_K, 300, 2048, 129),
    (O.Q6_K, 70, 256, 16),
    (O.Q4_1, 1024, 3072, 130),
    (O.BF16, 300, 1152, 77),
]


@pytest.mark.parametrize("fmt,rows,K,tokens", CASES)
def test_tiled_write_bit_exact(cuda, fmt, rows, K, tokens):
    rng = np.random.default_rng(rows * 7 + K + tokens + fmt)
    stored, piece, nb = weight(rng, fmt, rows, K)
    x = synth.activations(rng, tokens, K)
    y = torch.full((tokens, rows), float("nan"), dtype=torch.float32, device="cuda")
    run(fmt, K, [(dev(piece), nb, 0, rows, 0)], dev(x), [y])
    assert_exact(y.cpu().numpy(), O.matmul(fmt, piece, nb, rows, K, x))


def test_tiled_rows_equal_decoded_rows(cuda):
    """Batch invariance: each token of a 40-token step has the bits the decode
    form gives it alone (matmul.h 'Determinism')."""
    rng = np.random.default_rng(21)
    rows, K, T = 1500, 2048, 40
    stored, piece, nb = weight(rng, O.Q4_0, rows, K)
    x = synth.activations(rng, T, K)
    p, xd = dev(piece), dev(x)
    yT = torch.zeros((T, rows), dtype=torch.float32, device="cuda")
    run(O.Q4_0, K, [(p, nb, 0, rows, 0)], xd, [yT])
    for t in (0, 17, 39):
        y1 = torch.zeros((1, rows), dtype=torch.float32, device="cuda")
        run(O.Q4_0, K, [(p, nb, 0, rows, 0)], xd[t:t + 1], [y1], flags=0)
        assert_exact(yT[t].cpu().numpy(), y1.cpu().numpy())


def test_tiled_qkv_members_straddling_tiles(cuda):
    """Members whose rows are not tile multiples: a tile holds rows of two
    members, each landing in its own buffer at its stride."""
    rng = np.random.default_rng(5)
    K, T = 1024, 70
    x = synth.activations(rng, T, K)
    members, wants, outs = [], [], []
    for rows in (200, 90, 90):
        stored, piece, nb = weight(rng, O.Q4_0, rows, K)
        members.append((dev(piece), nb, 0, rows, 0))
        wants.append(O.matmul(O.Q4_0, piece, nb, rows, K, x))
        outs.append(torch.zeros((T, rows), dtype=torch.float32, device="cuda"))
    run(O.Q4_0, K, members, dev(x), outs, epilogue=cb.QKV)
    for o, w in zip(outs, wants):
        assert_exact(o.cpu().numpy(), w)


@pytest.mark.parametrize("activation", [cb.SILU, cb.GELU_TANH])
@pytest.mark.parametrize("F,T", [(3072, 512), (100, 20)])
def test_tiled_gated(cuda, activation, F, T):
    rng = np.random.default_rng(F + T + activation)
    K = 1024
    gs, gp, gnb = weight(rng, O.Q4_0, F, K)
    us, up, unb = weight(rng, O.Q4_0, F, K)
    x = synth.activations(rng, T, K) * 4
    y = torch.zeros((T, F), dtype=torch.float32, device="cuda")
    run(O.Q4_0, K, [(dev(gp), gnb, 0, F, 0), (dev(up), unb, 0, F, 0)], dev(x), [y], epilogue=cb.GATED,
        activation=activation)
    gate = O.matmul(O.Q4_0, gp, gnb, F, K, x)
    upv = O.matmul(O.Q4_0, up, unb, F, K, x)
    assert_exact(y.cpu().numpy(), (act_of(activation, gate) * upv).astype(np.float32))


def test_tiled_gate_and_up_as_halves_of_one_piece(cuda):
    """The fused gate|up piece of a Gemma-style model: both members read one
    piece, the up rows from first_row = F."""
    rng = np.random.default_rng(9)
    F, K, T = 600, 1152, 48
    stored, piece, nb = weight(rng, O.Q8_0, 2 * F, K)
    x = synth.activations(rng, T, K)
    p = dev(piece)
    y = torch.zeros((T, F), dtype=torch.float32, device="cuda")
    run(O.Q8_0, K, [(p, nb, 0, F, 0), (p, nb, F, F, 0)], dev(x), [y], epilogue=cb.GATED,
        activation=cb.GELU_TANH)
    both = O.matmul(O.Q8_0, piece, nb, 2 * F, K, x)
    assert_exact(y.cpu().numpy(), (act_of(cb.GELU_TANH, both[:, :F]) * both[:, F:]).astype(np.float32))


def test_tiled_gated_by_input(cuda):
    rng = np.random.default_rng(8)
    rows, K, T = 640, 1024, 24
    stored, piece, nb = weight(rng, O.Q4_0, rows, K)
    x = synth.activations(rng, T, K)
    u = rng.standard_normal((T + 3, 1000)).astype(np.float32)
    y = torch.zeros((T, rows), dtype=torch.float32, device="cuda")
    run(O.Q4_0, K, [(dev(piece), nb, 0, rows, 0)], dev(x), [y], epilogue=cb.GATED_BY_INPUT,
        activation=cb.SILU, gate_input=dev(u), gate_input_stride=1000, gate_input_column=100,
        gate_input_token=2)
    t = O.matmul(O.Q4_0, piece, nb, rows, K, x)
    assert_exact(y.cpu().numpy(), act_of(cb.SILU, t) * u[2:2 + T, 100:100 + rows])


def test_tiled_strided_input_and_output(cuda):
    """x rows and y rows at strides wider than the product (rows of a larger
    working buffer), with the output written at a column offset."""
    rng = np.random.default_rng(31)
    rows, K, T = 500, 1024, 33
    stored, piece, nb = weight(rng, O.Q6_K, rows, K)
    xw = synth.activations(rng, T, K + 64)
    y = torch.zeros((T, rows + 100), dtype=torch.float32, device="cuda")
    cb.matmul(O.Q6_K, K, [(dev(piece), nb, 0, rows, 100)], dev(xw), [y], x_stride=K + 64,
              out_stride=[rows + 100, 0, 0], flags=cb.MATMUL_TILED)
    torch.cuda.synchronize()
    want = O.matmul(O.Q6_K, piece, nb, rows, K, np.ascontiguousarray(xw[:, :K]))
    got = y.cpu().numpy()
    assert_exact(got[:, 100:], want)
    assert not got[:, :100].any()
