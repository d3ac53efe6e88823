"""An encoder's kernels (src/core/graph/encoder.h: EmbeddingGemma 2's text
encoder) against the oracle: the norm's encoder variants (norm.h:69-82 —
a scaled add, an add alone, several rows a token, no gain), rope's encode
form (rope_encode.wgsl: keys turned in place, values normalized), block
attention (block_attention.wgsl scores_of + weigh) and pooling (pool.wgsl
mean and unit).

Parity tier: bit-exact — every output equals the oracle's restatement of
the reference's order of operations — at EmbeddingGemma 2's shapes (width
512 with 24 per-layer rows of 512 a token, heads of 256 and 512, a window
of 512 either side halved) and at the edges the reference's tests name
(steps of 1, 2, 17, 33 and 512 rows; a window shorter than the step; rows
of zeros, tiny and large values)."""
import numpy as np
import pytest
import torch

import charlotte_b200 as cb
import oracle as O

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def done():
    torch.cuda.synchronize()
    cb.check(cb.lib().cb_fault_check(None))


def same(got, want):
    np.testing.assert_array_equal(np.asarray(got).view(np.uint32), np.asarray(want, np.float32).view(np.uint32))


# ---- norm variants -------------------------------------------------------------

@pytest.mark.parametrize("width,tokens", [(512, 5), (1152, 3), (2048, 1)])
@pytest.mark.parametrize("post", [False, True])
def test_norm_scaled_add(cuda, width, tokens, post):
    """Gemma 4's layer output scale: x = (x + postnorm(y))·s, then normed."""
    rng = np.random.default_rng(width + tokens + post)
    x = rng.standard_normal((tokens, width)).astype(np.float32)
    y = rng.standard_normal((tokens, width)).astype(np.float32)
    g = (rng.random(width) + 0.5).astype(np.float32)
    pg = (rng.random(width) + 0.5).astype(np.float32) if post else None
    s = np.array([0.37], np.float32)
    hidden, normed = dev(x), torch.zeros((tokens, width), dtype=torch.float32, device="cuda")
    cb.run("norm", hidden=hidden, output=dev(y), gain=dev(g), post_gain=dev(pg) if post else None, normed=normed,
           width=width, tokens=tokens, add=1, epsilon=1e-6, scale=dev(s))
    done()
    for t in range(tokens):
        h, n = O.norm_row_ex(x[t], y[t], g, epsilon=1e-6, post_gain=pg, scale=s)
        same(hidden[t].cpu().numpy(), h)
        same(normed[t].cpu().numpy(), n)


def test_norm_add_alone_leaves_normed(cuda):
    """normalize = false: X written after the add, nothing else."""
    rng = np.random.default_rng(3)
    width, tokens = 512, 4
    x = rng.standard_normal((tokens, width)).astype(np.float32)
    y = rng.standard_normal((tokens, width)).astype(np.float32)
    pg = (rng.random(width) + 0.5).astype(np.float32)
    hidden = dev(x)
    normed = torch.full((tokens, width), 7.0, dtype=torch.float32, device="cuda")
    cb.run("norm", hidden=hidden, output=dev(y), gain=dev(pg), post_gain=dev(pg), normed=normed, width=width,
           tokens=tokens, add=1, epsilon=1e-6, add_only=1)
    done()
    assert bool((normed == 7.0).all())
    for t in range(tokens):
        h, _ = O.norm_row_ex(x[t], y[t], pg, epsilon=1e-6, post_gain=pg, normalize=False)
        same(hidden[t].cpu().numpy(), h)


@pytest.mark.parametrize("rows_per_token,tokens", [(24, 3), (2, 2), (26, 1)])
def test_norm_rows_per_token(cuda, rows_per_token, tokens):
    """The per-layer inputs: each 512-wide slice of a token its own row, with
    ε × W (the projection's 1/√W folded in)."""
    rng = np.random.default_rng(rows_per_token * 7 + tokens)
    width = 512
    x = (rng.standard_normal((tokens * rows_per_token, width)) * 3).astype(np.float32)
    g = (rng.random(width) + 0.5).astype(np.float32)
    eps = np.float32(1e-6 * 768)
    hidden, normed = dev(x), torch.zeros_like(dev(x))
    cb.run("norm", hidden=hidden, output=None, gain=dev(g), post_gain=None, normed=normed, width=width,
           tokens=tokens, add=0, epsilon=float(eps), rows_per_token=rows_per_token)
    done()
    got = normed.cpu().numpy()
    for r in range(tokens * rows_per_token):
        _, n = O.norm_row_ex(x[r], None, g, epsilon=float(eps), add=False)
        same(got[r], n)


def test_norm_unit_gain(cuda):
    rng = np.random.default_rng(5)
    width, tokens = 1536, 3
    x = rng.standard_normal((tokens, width)).astype(np.float32)
    normed = torch.zeros((tokens, width), dtype=torch.float32, device="cuda")
    cb.run("norm", hidden=dev(x), output=None, gain=None, post_gain=None, normed=normed, width=width, tokens=tokens,
           add=0, epsilon=1e-6)
    done()
    for t in range(tokens):
        _, n = O.norm_row_ex(x[t], None, None, epsilon=1e-6, add=False)
        same(normed[t].cpu().numpy(), n)


# ---- rope's encode form ----------------------------------------------------------

ROPE = [
    # d, Hq, Hkv, halves, qk_norm, value_norm
    (256, 4, 1, True, True, True),     # EmbeddingGemma 2's sliding layers
    (512, 4, 1, True, True, True),     # its global layers: a head's 64 lanes over two warps
    (256, 4, 1, True, True, False),
    (128, 16, 8, True, False, True),
    (64, 32, 8, False, True, True),
]


@pytest.mark.parametrize("case", ROPE, ids=[f"d{c[0]}_{c[1]}x{c[2]}_h{int(c[3])}_qk{int(c[4])}_vn{int(c[5])}"
                                            for c in ROPE])
def test_rope_encode_form(cuda, case):
    d, hq, hkv, halves, qk, vn = case
    rng = np.random.default_rng(d + hq + hkv + 2 * qk + vn)
    tokens = 37
    turns = O.rope_turns(10000.0, d)
    qg = (rng.random(d) + 0.5).astype(np.float32) if qk else None
    kg = (rng.random(d) + 0.5).astype(np.float32) if qk else None
    q = (rng.standard_normal((tokens, hq * d)) * 2).astype(np.float32)
    k = (rng.standard_normal((tokens, hkv * d)) * 2).astype(np.float32)
    v = (rng.standard_normal((tokens, hkv * d)) * 2).astype(np.float32)
    qd, kd, vd = dev(q), dev(k), dev(v)
    cb.run("rope", query=qd, key=kd, value=vd, key_cache=None, value_cache=None, query_gain=dev(qg) if qk else None,
           key_gain=dev(kg) if qk else None, factors=None, turns=dev(turns), position=None, position0=0,
           tokens=tokens, head_dim=d, query_heads=hq, kv_heads=hkv, halves=int(halves), slots=0, epsilon=1e-6,
           encode=1, value_norm=int(vn))
    done()
    for t in (0, 1, 17, tokens - 1):
        qq, kk, vv = q[t].copy(), k[t].copy(), v[t].copy()
        O.rope_encode_token(qq, kk, vv, t, head_dim=d, query_heads=hq, kv_heads=hkv, halves=halves, epsilon=1e-6,
                            turns=turns, query_gain=qg, key_gain=kg, value_norm=vn)
        same(qd[t].cpu().numpy(), qq)
        same(kd[t].cpu().numpy(), kk)
        same(vd[t].cpu().numpy(), vv)


# ---- block attention -------------------------------------------------------------

BLOCK = [
    # d, Hq, Hkv, half_window, tokens
    (256, 4, 1, 256, 512),     # EmbeddingGemma 2's sliding layer, a 512-token step
    (512, 4, 1, 1 << 20, 130),  # its global layer (the trained context's window)
    (256, 4, 2, 16, 77),       # a window shorter than the step
    (64, 8, 8, 1 << 20, 33),
    (128, 16, 1, 5, 17),
    (256, 4, 1, 256, 1),
    (256, 2, 1, 256, 2),
]


@pytest.mark.parametrize("case", BLOCK, ids=[f"d{c[0]}_{c[1]}x{c[2]}_h{min(c[3], 9999)}_n{c[4]}" for c in BLOCK])
def test_block_attention_bit_exact(cuda, case):
    d, hq, hkv, half, n = case
    rng = np.random.default_rng(d + hq + n + half % 97)
    q = rng.standard_normal((n, hq * d)).astype(np.float32)
    k = rng.standard_normal((n, hkv * d)).astype(np.float32)
    v = rng.standard_normal((n, hkv * d)).astype(np.float32)
    scale = float(np.float32(1.4426950408889634))   # EmbeddingGemma 2's scale of 1, in log2 units
    out = torch.full((n, hq * d), float("nan"), dtype=torch.float32, device="cuda")
    cb.run("block_attention", query=dev(q), key=dev(k), value=dev(v), out=out, tokens=n, head_dim=d, query_heads=hq,
           kv_heads=hkv, half_window=half, scale_log2e=scale)
    done()
    want = O.block_attention(q, k, v, tokens=n, head_dim=d, query_heads=hq, kv_heads=hkv, half_window=half,
                             scale_log2e=scale)
    same(out.cpu().numpy(), want)


def test_block_attention_refuses_what_does_not_fit(cuda):
    q = torch.zeros((2048, 4 * 512), dtype=torch.float32, device="cuda")
    k = torch.zeros((2048, 512), dtype=torch.float32, device="cuda")
    with pytest.raises(cb.CharlotteError):
        cb.run("block_attention", query=q, key=k, value=k, out=q, tokens=2048, head_dim=512, query_heads=4,
               kv_heads=1, half_window=256, scale_log2e=1.0)
    with pytest.raises(cb.CharlotteError):   # 3 query heads a kv head do not divide 16
        cb.run("block_attention", query=q, key=k, value=k, out=q, tokens=4, head_dim=64, query_heads=3,
               kv_heads=1, half_window=4, scale_log2e=1.0)


# ---- pooling -----------------------------------------------------------------------

@pytest.mark.parametrize("n", [1, 2, 33, 512])
def test_pool_mean_written_at_the_last_row(cuda, n):
    rng = np.random.default_rng(n)
    width = 512
    rows = rng.standard_normal((n, width)).astype(np.float32)
    out = torch.full((n, width), 5.0, dtype=torch.float32, device="cuda")
    cb.run("pool", input=dev(rows), output=out, width=width, tokens=n, kind=cb.POOL_MEAN)
    done()
    got = out.cpu().numpy()
    same(got[n - 1], O.pool_mean(rows))
    assert (got[:n - 1] == 5.0).all()


@pytest.mark.parametrize("scale", [1e18, 1e-18, 0.0, 1.0])
def test_pool_unit(cuda, scale):
    rng = np.random.default_rng(7)
    for width in (768, 4096, 12):
        row = (rng.standard_normal(width) * scale).astype(np.float32)
        out = torch.full((width,), 3.0, dtype=torch.float32, device="cuda")
        cb.run("pool", input=dev(row), output=out, width=width, tokens=1, kind=cb.POOL_UNIT)
        done()
        same(out.cpu().numpy(), O.pool_unit(row))
