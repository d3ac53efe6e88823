"""The tensor-core form of the matrix products (CB_MATMUL_TENSOR: tcgen05
MMA, f16 operands, f32 accumulation in tensor memory) against f64 products
over the reference's own dequantized weights.

Parity tier: tolerance, as BASELINE states it for GEMV/GEMM outputs and
logits: max |y - y_f64| <= 1e-3 * max |y_f64| (TOL below). The weights are
decoded exactly first (the same decode the exact forms use), then rounded to
f16 with x. Cases cover each format, each epilogue, ragged token and row
tails (partial 128-token and 128-slot tiles), a K that ends in half a
64-wide block, and a step long enough to cycle the 4-stage ring many times."""
import ctypes

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


FORMS = ["fused", "dense"]


def run(fmt, K, members, x, outs, form="fused", **kw):
    """The tensor form; `dense`: the weights densified first (cb_matmul_densify)
    and scratch with room for eight splits of K after x16."""
    if form == "dense":
        kw["dense"] = cb.densify(fmt, K, members, epilogue=kw.get("epilogue", cb.WRITE),
                                 activation=kw.get("activation", cb.SILU))
        tokens = x.shape[0]
        slots = sum(m[3] for m in members) + 128
        n = cb.lib().cb_matmul_scratch_bytes(cb.MATMUL_TENSOR, tokens, K) + 8 * tokens * slots * 4
        kw["scratch"] = torch.empty(n, dtype=torch.uint8, device="cuda")
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


@pytest.mark.parametrize("form", FORMS)
@pytest.mark.parametrize("fmt,rows,K,tokens", CASES)
def test_tensor_write_within_tolerance(cuda, fmt, rows, K, tokens, form):
    rng = np.random.default_rng(rows + K * 3 + tokens + fmt)
    stored, piece, nb = weight(rng, fmt, rows, K)
    x = synth.activations(rng, tokens, K)
    y = torch.full((tokens, rows), float("nan"), dtype=torch.float32, device="cuda")
    run(fmt, K, [(dev(piece), nb, 0, rows, 0)], dev(x), [y], form=form)
    within(y.cpu().numpy(), exact(fmt, stored, rows, K, x))


# Few tiles over a wide K: the dense form splits K (partials added in split
# order by a second launch); a product of many tiles takes N = 256 tiles.
@pytest.mark.parametrize("fmt,rows,K,tokens", [(O.Q4_0, 2048, 8192, 512), (O.Q4_0, 1024, 2048, 200),
                                               (O.Q8_0, 640, 6912, 64), (O.Q4_0, 16384, 1024, 512)])
def test_dense_split_and_wide_tiles(cuda, fmt, rows, K, tokens):
    rng = np.random.default_rng(rows + K + tokens)
    stored, piece, nb = weight(rng, fmt, rows, K)
    x = synth.activations(rng, tokens, K)
    y = torch.full((tokens, rows), float("nan"), dtype=torch.float32, device="cuda")
    run(fmt, K, [(dev(piece), nb, 0, rows, 0)], dev(x), [y], form="dense")
    within(y.cpu().numpy(), exact(fmt, stored, rows, K, x))
    # without room for partials: one split, the same sums to within the tier
    z = torch.full_like(y, float("nan"))
    members = [(dev(piece), nb, 0, rows, 0)]
    dense = cb.densify(fmt, K, members)
    cb.matmul(fmt, K, members, dev(x), [z], flags=cb.MATMUL_TENSOR, dense=dense)
    torch.cuda.synchronize()
    within(z.cpu().numpy(), exact(fmt, stored, rows, K, x))


def q6_k_weights(stored, rows, K):
    """The f32 weights of Q6_K blocks as the products' decode forms them:
    s = d·sc, then fma(1 + q/128, 128·s, -160·s) (the magic-float decode).
    s has at most 19 significant bits, so every step is exact and the value
    is the reference dequantizer's s·(q - 32) — except that a zero weight is
    +0 here where s·0 keeps the sign of s."""
    blk = stored.reshape(-1, 210)
    d = blk[:, 208:210].copy().view(np.float16).astype(np.float32)[:, 0]
    out = np.empty((blk.shape[0], 256), np.float32)
    for k in range(8):
        h, r = k // 4, k % 4
        for l in range(32):
            lo = (blk[:, 64 * h + 32 * (r % 2) + l] >> (4 * (r // 2))) & 0xF
            hi = (blk[:, 128 + 32 * h + l] >> (2 * r)) & 3
            q = (lo | (hi << 4)).astype(np.float64)
            sc = blk[:, 192 + 2 * k + l // 16].view(np.int8).astype(np.float32)
            s = (d * sc).astype(np.float32)
            S = (s * np.float32(128)).astype(np.float64)
            C = (s * np.float32(-160)).astype(np.float32).astype(np.float64)
            out[:, 32 * k + l] = ((1.0 + q / 128.0) * S + C).astype(np.float32)
    return out.reshape(rows, K)


@pytest.mark.parametrize("fmt", [O.Q4_0, O.Q8_0, O.Q6_K, O.Q4_1, O.BF16])
def test_densified_weights_are_the_decoded_weights_rounded_to_f16(cuda, fmt):
    """Bit-exact: each dense row is its weight row as the exact forms decode
    it (the reference's dequantizers; Q6_K its magic-float form), rounded to
    f16 (nearest even); a gated product's rows interleave 64-row units of
    gate and up rows, zero rows padding the last pair."""
    rng = np.random.default_rng(fmt + 5)
    K = 512
    gs, gp, gnb = weight(rng, fmt, 100, K)
    us, up, unb = weight(rng, fmt, 100, K)
    if fmt == O.Q6_K:
        G = q6_k_weights(gs, 100, K).astype(np.float16)
        U = q6_k_weights(us, 100, K).astype(np.float16)
    else:
        G = O.dequant_stored(fmt, gs).reshape(100, K).astype(np.float16)
        U = O.dequant_stored(fmt, us).reshape(100, K).astype(np.float16)
    members = [(dev(gp), gnb, 0, 100, 0), (dev(up), unb, 0, 100, 0)]
    d = cb.densify(fmt, K, members, epilogue=cb.GATED).cpu().numpy().view(np.float16).reshape(-1, K)
    assert d.shape[0] == 256
    for unit in range(4):
        src = G if unit % 2 == 0 else U
        lo = (unit // 2) * 64
        n = min(64, 100 - lo)
        np.testing.assert_array_equal(d[unit * 64: unit * 64 + n].view(np.uint16), src[lo:lo + n].view(np.uint16))
        assert not d[unit * 64 + n: unit * 64 + 64].any()
    # members one after another, a member's first row honoured
    d2 = cb.densify(fmt, K, [(dev(gp), gnb, 10, 50, 0), (dev(up), unb, 0, 30, 0)],
                    epilogue=cb.QKV).cpu().numpy().view(np.float16).reshape(-1, K)
    np.testing.assert_array_equal(d2.view(np.uint16), np.concatenate([G[10:60], U[:30]]).view(np.uint16))


@pytest.mark.parametrize("form", FORMS)
def test_tensor_qkv(cuda, form):
    rng = np.random.default_rng(41)
    K, T = 1024, 300
    x = synth.activations(rng, T, K)
    members, wants, outs = [], [], []
    for rows in (2048, 1000, 1000):
        stored, piece, nb = weight(rng, O.Q4_0, rows, K)
        members.append((dev(piece), nb, 0, rows, 0))
        wants.append(exact(O.Q4_0, stored, rows, K, x))
        outs.append(torch.zeros((T, rows), dtype=torch.float32, device="cuda"))
    run(O.Q4_0, K, members, dev(x), outs, epilogue=cb.QKV, form=form)
    for o, w in zip(outs, wants):
        within(o.cpu().numpy(), w)


@pytest.mark.parametrize("form", FORMS)
@pytest.mark.parametrize("activation", [cb.SILU, cb.GELU_TANH])
def test_tensor_gated(cuda, activation, form):
    rng = np.random.default_rng(43 + activation)
    F, K, T = 3000, 1024, 257
    gs, gp, gnb = weight(rng, O.Q4_0, F, K)
    us, up, unb = weight(rng, O.Q4_0, F, K)
    x = synth.activations(rng, T, K)
    y = torch.zeros((T, F), dtype=torch.float32, device="cuda")
    run(O.Q4_0, K, [(dev(gp), gnb, 0, F, 0), (dev(up), unb, 0, F, 0)], dev(x), [y], epilogue=cb.GATED,
        activation=activation, form=form)
    g = exact(O.Q4_0, gs, F, K, x)
    u = exact(O.Q4_0, us, F, K, x)
    if activation == cb.SILU:
        act = g / (1.0 + np.exp(-g))
    else:
        act = 0.5 * g * (1.0 + np.tanh(0.7978845608028654 * (g + 0.044715 * g ** 3)))
    within(y.cpu().numpy(), act * u)


@pytest.mark.parametrize("form", FORMS)
def test_tensor_gated_by_input(cuda, form):
    rng = np.random.default_rng(47)
    rows, K, T = 640, 1024, 150
    stored, piece, nb = weight(rng, O.Q4_0, rows, K)
    x = synth.activations(rng, T, K)
    u = rng.standard_normal((T + 3, 1000)).astype(np.float32)
    y = torch.zeros((T, rows), dtype=torch.float32, device="cuda")
    run(O.Q4_0, K, [(dev(piece), nb, 0, rows, 0)], dev(x), [y], epilogue=cb.GATED_BY_INPUT,
        activation=cb.SILU, gate_input=dev(u), gate_input_stride=1000, gate_input_column=100,
        gate_input_token=2, form=form)
    t = exact(O.Q4_0, stored, rows, K, x)
    within(y.cpu().numpy(), t / (1.0 + np.exp(-t)) * u[2:2 + T, 100:100 + rows])


def test_dense_reads_x16_and_writes_out16(cuda):
    """A producer's f16 copy of x (cb_matmul.x16) gives the bits of x rounded
    by the product itself; a gated product's out16 is its output rounded to
    f16 (the next product's x16)."""
    rng = np.random.default_rng(53)
    F, K, T = 2048, 1024, 300
    gs, gp, gnb = weight(rng, O.Q4_0, F, K)
    us, up, unb = weight(rng, O.Q4_0, F, K)
    x = synth.activations(rng, T, K)
    members = [(dev(gp), gnb, 0, F, 0), (dev(up), unb, 0, F, 0)]
    dense = cb.densify(O.Q4_0, K, members, epilogue=cb.GATED)
    n = cb.lib().cb_matmul_scratch_bytes(cb.MATMUL_TENSOR, T, K) + 8 * T * 2 * F * 4
    scratch = torch.empty(n, dtype=torch.uint8, device="cuda")
    y0 = torch.zeros((T, F), dtype=torch.float32, device="cuda")
    cb.matmul(O.Q4_0, K, members, dev(x), [y0], epilogue=cb.GATED, flags=cb.MATMUL_TENSOR, scratch=scratch,
              dense=dense)
    x16 = dev(x).half()
    y1 = torch.zeros_like(y0)
    o16 = torch.zeros((T, F), dtype=torch.float16, device="cuda")
    m = cb._product(O.Q4_0, K, members, cb.GATED, cb.SILU)
    m.scratch, m.scratch_bytes, m.dense = scratch.data_ptr(), n, dense.data_ptr()
    m.x16, m.out16 = x16.data_ptr(), o16.data_ptr()
    outs = (ctypes.c_void_p * 3)(y1.data_ptr(), None, None)
    strides = (ctypes.c_uint32 * 3)(F, 0, 0)
    cb.check(cb.lib().cb_matmul_run(ctypes.byref(m), dev(x).data_ptr(), K, T, ctypes.byref(outs),
                                    ctypes.byref(strides), cb.MATMUL_TENSOR, None))
    torch.cuda.synchronize()
    assert torch.equal(y0, y1)
    assert torch.equal(o16, y1.half())
