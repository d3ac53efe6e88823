"""The split form of the matrix products (matmul.wgsl split_ranges :609 and
combine_* :651-695; the split gate, matmul.h:637-646): the tiled form's
tiles once for each of the 32 ranges, each writing its range sums in the
reference's range_sums layout, then a combine adding each output's 32 in
order. Parity tier: bit-exact — every output equals the oracle's and the
other exact forms' — for every format, the Write, QKV and GatedByInput
epilogues (the reference never splits a gated product), ragged token and
row tails, ranges of one group and of many, and the widths where it is
chosen by size (Gemma's down product: 1,152 rows over K = 6,912)."""
import numpy as np
import pytest
import torch

import charlotte_b200 as cb
import oracle as O
from charlotte_b200 import synth

pytestmark = pytest.mark.gpu
SPLIT = cb.MATMUL_SPLIT


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def scratch(tokens, rows):
    n = cb.lib().cb_matmul_split_bytes(tokens, rows)
    return torch.zeros(n // 4, dtype=torch.float32, device="cuda")


def product(fmt, K, members, x, outs, flags, **kw):
    cb.matmul(fmt, K, members, x, outs, flags=flags, **kw)
    torch.cuda.synchronize()
    cb.check(cb.lib().cb_fault_check(None))


CASES = [
    (O.Q4_0, 1152, 6912, 64),   # Gemma's down, a 64-row batched step
    (O.Q4_0, 1152, 6912, 8),
    (O.Q4_0, 1024, 3072, 130),  # Qwen3's down, a ragged token tail
    (O.Q4_0, 1024, 2048, 512),  # Qwen3's O at a prefill block
    (O.Q4_0, 77, 2048, 9),      # ragged rows
    (O.Q8_0, 333, 6912, 33),
    (O.Q6_K, 300, 2048, 17),
    (O.Q4_1, 256, 4096, 40),
    (O.BF16, 128, 2048, 24),
    (O.Q4_0, 64, 1024, 5),      # one group a range
]


@pytest.mark.parametrize("fmt,rows,K,tokens", CASES)
def test_split_form_is_bit_exact(cuda, fmt, rows, K, tokens):
    rng = np.random.default_rng(rows * 7 + K + tokens)
    stored = synth.blocks(rng, fmt, rows, K)
    piece = synth.to_piece(fmt, stored)
    nb = rows * K // O.BLOCK_WEIGHTS[fmt]
    x = synth.activations(rng, tokens, K)
    want = O.matmul(fmt, piece, nb, rows, K, x)
    y = torch.zeros((tokens, rows), dtype=torch.float32, device="cuda")
    rs = scratch(tokens, rows)
    members = [(dev(piece), nb, 0, rows, 0)]
    product(fmt, K, members, dev(x), [y], cb.MATMUL_PDL | SPLIT, scratch=rs)
    np.testing.assert_array_equal(y.cpu().numpy(), want)
    # the range sums lie where the reference's range_sum_at puts them: each
    # output is its 32 sums added in order from zero
    sums = rs.cpu().numpy().reshape(32, tokens, rows)
    total = np.zeros((tokens, rows), np.float32)
    for r in range(32):
        total = (total + sums[r]).astype(np.float32)
    np.testing.assert_array_equal(total, want)
    # the same bits as the tiled and streamed forms
    for flags in (cb.MATMUL_TILED, cb.MATMUL_STREAMED):
        z = torch.zeros_like(y)
        product(fmt, K, members, dev(x), [z], flags)
        np.testing.assert_array_equal(z.cpu().numpy(), want)


def test_split_qkv_and_gated_input_epilogues(cuda):
    rng = np.random.default_rng(11)
    K, tokens = 2048, 48
    rows = [512, 128, 128]
    pieces, members = [], []
    for r in rows:
        st = synth.blocks(rng, O.Q4_0, r, K)
        pieces.append(synth.to_piece(O.Q4_0, st))
        members.append((dev(pieces[-1]), r * K // 32, 0, r, 0))
    x = synth.activations(rng, tokens, K)
    outs = [torch.zeros((tokens, r), dtype=torch.float32, device="cuda") for r in rows]
    product(O.Q4_0, K, members, dev(x), outs, SPLIT, epilogue=cb.QKV, scratch=scratch(tokens, sum(rows)))
    for o, p, r in zip(outs, pieces, rows):
        np.testing.assert_array_equal(o.cpu().numpy(), O.matmul(O.Q4_0, p, r * K // 32, r, K, x))
    # GatedByInput: act(y) * u at the token's row and the output's column
    u = rng.standard_normal((tokens, 600)).astype(np.float32)
    y = torch.zeros((tokens, 512), dtype=torch.float32, device="cuda")
    product(O.Q4_0, K, members[:1], dev(x), [y], SPLIT, epilogue=cb.GATED_BY_INPUT, activation=cb.GELU_TANH,
            gate_input=dev(u), gate_input_stride=600, gate_input_column=40, scratch=scratch(tokens, 512))
    base = O.matmul(O.Q4_0, pieces[0], 512 * K // 32, 512, K, x)
    act = np.vectorize(lambda g: O.lib().or_activate(cb.GELU_TANH, float(g)), otypes=[np.float32])(base)
    np.testing.assert_array_equal(y.cpu().numpy(), (act * u[:, 40:552]).astype(np.float32))


def test_split_refuses_gated_products_and_short_scratch(cuda):
    rng = np.random.default_rng(2)
    K, tokens = 2048, 16
    st = synth.blocks(rng, O.Q4_0, 256, K)
    p = dev(synth.to_piece(O.Q4_0, st))
    x = dev(synth.activations(rng, tokens, K))
    y = torch.zeros((tokens, 128), dtype=torch.float32, device="cuda")
    with pytest.raises(cb.CharlotteError) as e:
        cb.matmul(O.Q4_0, K, [(p, 256 * K // 32, 0, 128, 0), (p, 256 * K // 32, 128, 128, 0)], x, [y],
                  epilogue=cb.GATED, flags=SPLIT, scratch=scratch(tokens, 256))
    assert e.value.status == cb.ERROR_INVALID
    with pytest.raises(cb.CharlotteError) as e:
        cb.matmul(O.Q4_0, K, [(p, 256 * K // 32, 0, 256, 0)], x, [torch.zeros((tokens, 256), device="cuda")],
                  flags=SPLIT, scratch=scratch(tokens, 100))
    assert e.value.status == cb.ERROR_INVALID
