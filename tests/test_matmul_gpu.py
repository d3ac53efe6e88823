"""Matrix products on the GPU through the C ABI against the CPU oracle.

Parity tier: bit-exact. Every output of the decode form must equal the
oracle's — the reference's order of addition (matmul.h:34-50) restated in C —
bit for bit (zeros by value). The stated tolerance of the BASELINE tier,
max |y - y_f64| <= 1e-3 * max |y_f64|, is checked as well, against f64 over
the reference's own dequantized weights. Cases follow the reference's GPU
test plan (matmul.h 'Verification'): each format and epilogue, widths whose
ranges are one group, several, unequal, and mostly empty (K = 64), weights in
pieces, QKV outputs landing in their buffers, SiLU and GELU, and a token's
outputs identical alone or in a step of several."""
import numpy as np
import pytest
import torch

import charlotte_b200 as cb
import oracle as O
from charlotte_b200 import synth

pytestmark = pytest.mark.gpu

TOL = 1e-3   # BASELINE tier: max abs err <= 1e-3 * max |y|


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def weight(rng, fmt, rows, K, random_bytes=False):
    nb = rows * K // O.BLOCK_WEIGHTS[fmt]
    stored = synth.random_bytes_blocks(rng, fmt, nb) if random_bytes else synth.blocks(rng, fmt, rows, K)
    return stored, synth.to_piece(fmt, stored), nb


def run(fmt, K, members, x, outs, **kw):
    cb.matmul(fmt, K, members, x, outs, **kw)
    torch.cuda.synchronize()
    cb.check(cb.lib().cb_fault_check(None))   # no bounded wait ran out


def assert_exact(got, want):
    """Bit-exact (zeros by value); a NaN must meet a NaN (weights of random
    bytes reach every exponent, so sums can overflow to inf − inf)."""
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    g, w = got.reshape(-1), want.reshape(-1)
    bad = np.flatnonzero((g != w) & ~(np.isnan(g) & np.isnan(w)))
    assert bad.size == 0, f"{bad.size} outputs differ; first at {bad[:5]}: {got.reshape(-1)[bad[:5]]} vs {want.reshape(-1)[bad[:5]]}"


def assert_tolerance(got, stored, fmt, rows, K, x):
    W = O.dequant_stored(fmt, stored).reshape(rows, K).astype(np.float64)
    exact = x.astype(np.float64) @ W.T
    err = np.max(np.abs(got.astype(np.float64) - exact))
    assert err <= TOL * np.max(np.abs(exact)), (err, np.max(np.abs(exact)))


SHAPES = [
    (O.Q4_0, 8192, 2048),    # config 1, Llama-3.2-1B gate_proj
    (O.Q4_0, 4096, 1024),    # Qwen3 QKV
    (O.Q4_0, 1024, 3072),    # Qwen3 down: 3 groups a range
    (O.Q4_0, 1152, 6912),    # Gemma 3 down: unequal ranges
    (O.Q4_0, 100, 1152),     # Gemma 3 width: 36 groups
    (O.Q4_0, 77, 64),        # 2 groups: 30 ranges empty
    (O.Q8_0, 1024, 1024),
    (O.Q8_0, 333, 6912),
    (O.Q8_0, 50, 64),
    (O.Q6_K, 4096, 1024),    # the Qwen3 head's shape, fewer rows
    (O.Q6_K, 300, 2048),
    (O.Q6_K, 70, 6912),
    (O.Q6_K, 31, 256),
    (O.Q4_1, 1024, 3072),    # the Qwen3 file's Q4_1 down projection
    (O.Q4_1, 100, 1152),
    (O.BF16, 1024, 1024),
    (O.BF16, 77, 64),
]


@pytest.mark.parametrize("fmt,rows,K", SHAPES)
def test_decode_write_bit_exact(cuda, fmt, rows, K):
    rng = np.random.default_rng(rows * 31 + K + fmt)
    stored, piece, nb = weight(rng, fmt, rows, K)
    x = synth.activations(rng, 1, K)
    y = torch.zeros((1, rows), dtype=torch.float32, device="cuda")
    run(fmt, K, [(dev(piece), nb, 0, rows, 0)], dev(x), [y])
    want = O.matmul(fmt, piece, nb, rows, K, x)
    got = y.cpu().numpy()
    assert_exact(got, want)
    assert_tolerance(got, stored, fmt, rows, K, x)


@pytest.mark.parametrize("fmt", [O.Q4_0, O.Q4_1, O.Q8_0, O.Q6_K, O.BF16])
def test_dequant_through_one_hot_inputs_is_bit_exact(cuda, fmt):
    """x = e_k gives y[o] = w[o][k] exactly (one fma of w by 1 onto +0), so
    K one-hot tokens read the whole decoded matrix back: every weight must
    equal the reference's dequantizer's, over random bytes (all code and scale
    classes, subnormal scales included)."""
    rng = np.random.default_rng(fmt)
    rows, K = 40, 256
    stored, piece, nb = weight(rng, fmt, rows, K, random_bytes=True)
    x = np.eye(K, dtype=np.float32)
    y = torch.zeros((K, rows), dtype=torch.float32, device="cuda")
    run(fmt, K, [(dev(piece), nb, 0, rows, 0)], dev(x), [y])
    W = O.dequant_stored(fmt, stored).reshape(rows, K)
    assert_exact(y.cpu().numpy().T, W)


@pytest.mark.parametrize("fmt", [O.Q4_0, O.Q4_1, O.Q6_K, O.BF16])
def test_random_bytes_weights_bit_exact(cuda, fmt):
    rng = np.random.default_rng(77 + fmt)
    rows, K = 257, 2048
    stored, piece, nb = weight(rng, fmt, rows, K, random_bytes=True)
    x = synth.activations(rng, 1, K)
    y = torch.zeros((1, rows), dtype=torch.float32, device="cuda")
    run(fmt, K, [(dev(piece), nb, 0, rows, 0)], dev(x), [y])
    assert_exact(y.cpu().numpy(), O.matmul(fmt, piece, nb, rows, K, x))


def test_qkv_members_land_in_their_buffers(cuda):
    rng = np.random.default_rng(3)
    K = 1024
    parts = [(2048, None), (1024, None), (1024, None)]
    members, wants, outs = [], [], []
    x = synth.activations(rng, 1, K)
    for rows, _ in parts:
        stored, piece, nb = weight(rng, O.Q4_0, rows, K)
        members.append((dev(piece), nb, 0, rows, 0))
        wants.append(O.matmul(O.Q4_0, piece, nb, rows, K, x))
        outs.append(torch.zeros((1, rows), dtype=torch.float32, device="cuda"))
    run(O.Q4_0, K, members, dev(x), outs, epilogue=cb.QKV)
    for o, w in zip(outs, wants):
        assert_exact(o.cpu().numpy(), w)


@pytest.mark.parametrize("activation", [cb.SILU, cb.GELU_TANH])
@pytest.mark.parametrize("F", [3072, 100])
def test_gated_activation(cuda, activation, F):
    rng = np.random.default_rng(F + activation)
    K = 1024
    gs, gp, gnb = weight(rng, O.Q4_0, F, K)
    us, up, unb = weight(rng, O.Q4_0, F, K)
    x = synth.activations(rng, 1, K) * 4
    y = torch.zeros((1, F), dtype=torch.float32, device="cuda")
    run(O.Q4_0, K, [(dev(gp), gnb, 0, F, 0), (dev(up), unb, 0, F, 0)], dev(x), [y], epilogue=cb.GATED,
        activation=activation)
    gate = O.matmul(O.Q4_0, gp, gnb, F, K, x)[0]
    upv = O.matmul(O.Q4_0, up, unb, F, K, x)[0]
    act = np.array([O.lib().or_activate(activation, float(g)) for g in gate], np.float32)
    assert_exact(y.cpu().numpy()[0], (act * upv).astype(np.float32))


def test_gated_by_input(cuda):
    rng = np.random.default_rng(8)
    rows, K = 640, 1024
    stored, piece, nb = weight(rng, O.Q4_0, rows, K)
    x = synth.activations(rng, 1, K)
    u = rng.standard_normal((3, 1000)).astype(np.float32)
    y = torch.zeros((1, rows), dtype=torch.float32, device="cuda")
    run(O.Q4_0, K, [(dev(piece), nb, 0, rows, 0)], dev(x), [y], epilogue=cb.GATED_BY_INPUT,
        activation=cb.GELU_TANH, gate_input=dev(u), gate_input_stride=1000, gate_input_column=100,
        gate_input_token=2)
    t = O.matmul(O.Q4_0, piece, nb, rows, K, x)[0]
    want = np.array([O.lib().or_activate(cb.GELU_TANH, float(v)) for v in t], np.float32) * u[2, 100:100 + rows]
    assert_exact(y.cpu().numpy()[0], want)


def test_tokens_step_invariance(cuda):
    """A token's outputs are the same bits decoded alone or in a step of 7."""
    rng = np.random.default_rng(12)
    rows, K = 1000, 3072
    stored, piece, nb = weight(rng, O.Q4_0, rows, K)
    x = synth.activations(rng, 7, K)
    p = dev(piece)
    y7 = torch.zeros((7, rows), dtype=torch.float32, device="cuda")
    run(O.Q4_0, K, [(p, nb, 0, rows, 0)], dev(x), [y7])
    for t in range(7):
        y1 = torch.zeros((1, rows), dtype=torch.float32, device="cuda")
        run(O.Q4_0, K, [(p, nb, 0, rows, 0)], dev(x[t:t + 1]), [y1])
        assert_exact(y7[t:t + 1].cpu().numpy(), y1.cpu().numpy())
    assert_exact(y7.cpu().numpy(), O.matmul(O.Q4_0, piece, nb, rows, K, x))


def test_weight_in_pieces_with_output_offsets(cuda):
    """A head split by rows into pieces, one launch a piece, each writing its
    rows' columns (matmul.h 'Pieces')."""
    rng = np.random.default_rng(14)
    K = 1024
    x = synth.activations(rng, 1, K)
    y = torch.zeros((1, 700), dtype=torch.float32, device="cuda")
    wants = []
    first = 0
    for rows in (300, 400):
        stored, piece, nb = weight(rng, O.Q6_K, rows, K)
        run(O.Q6_K, K, [(dev(piece), nb, 0, rows, first)], dev(x), [y])
        wants.append(O.matmul(O.Q6_K, piece, nb, rows, K, x)[0])
        first += rows
    assert_exact(y.cpu().numpy()[0], np.concatenate(wants))


def test_pdl_launch_matches(cuda):
    rng = np.random.default_rng(15)
    rows, K = 2048, 1024
    stored, piece, nb = weight(rng, O.Q4_0, rows, K)
    x = synth.activations(rng, 1, K)
    y = torch.zeros((1, rows), dtype=torch.float32, device="cuda")
    p, xd = dev(piece), dev(x)
    for _ in range(3):
        run(O.Q4_0, K, [(p, nb, 0, rows, 0)], xd, [y], flags=cb.MATMUL_PDL)
    assert_exact(y.cpu().numpy(), O.matmul(O.Q4_0, piece, nb, rows, K, x))
