"""RMSNorm, QK-norm + RoPE + KV append, attention, gather and top-k/draw on
the GPU through the C ABI, against the CPU oracle. Parity tier: bit-exact
(zeros by value) — each kernel keeps the reference's order of operations and
the numerics definitions the oracle states. Attention is also held to a
stated tolerance against an f64 softmax (1e-4 relative to max |out|), the
norm to the reference's bound (norm.h:50-62: 2^-18 of the row's largest)."""
import math

import numpy as np
import pytest
import torch

import charlotte_b200 as cb
import oracle as O
from charlotte_b200 import synth

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def done():
    torch.cuda.synchronize()
    cb.check(cb.lib().cb_fault_check(None))


def same(got, want):
    got = np.asarray(got)
    want = np.asarray(want)
    if got.dtype == np.float32:
        bad = np.flatnonzero(got.reshape(-1) != want.reshape(-1))
    else:
        bad = np.flatnonzero(got.reshape(-1) != want.reshape(-1))
    assert bad.size == 0, f"{bad.size} differ, first {bad[:4]}: {got.reshape(-1)[bad[:4]]} vs {want.reshape(-1)[bad[:4]]}"


# ---- norm ---------------------------------------------------------------------

@pytest.mark.parametrize("width", [1024, 1152, 2048, 4096, 100])
@pytest.mark.parametrize("mode", ["plain", "add", "post"])
def test_norm_bit_exact(cuda, width, mode):
    rng = np.random.default_rng(width + len(mode))
    rows = 5
    hidden = (rng.standard_normal((rows, width)) * 3).astype(np.float32)
    out = rng.standard_normal((rows, width)).astype(np.float32)
    gain = (1 + 0.1 * rng.standard_normal(width)).astype(np.float32)
    post = (1 + 0.1 * rng.standard_normal(width)).astype(np.float32) if mode == "post" else None
    h, o, g = dev(hidden), dev(out), dev(gain)
    normed = torch.zeros((rows, width), dtype=torch.float32, device="cuda")
    cb.run("norm", hidden=h, output=o, gain=g, post_gain=dev(post) if post is not None else 0, normed=normed,
           width=width, tokens=rows, add=int(mode != "plain"), last_token=0, epsilon=1e-6)
    done()
    for r in range(rows):
        wh, wn = O.norm_row(hidden[r], out[r], gain, post, 1e-6, mode != "plain")
        same(h[r].cpu().numpy(), wh)
        same(normed[r].cpu().numpy(), wn)
        x64 = wh.astype(np.float64)
        exact = x64 / np.sqrt(np.mean(x64 * x64) + 1e-6) * gain
        assert np.max(np.abs(normed[r].cpu().numpy() - exact)) <= 2.0 ** -18 * np.max(np.abs(exact)) * 4


def test_norm_last_token_only(cuda):
    rng = np.random.default_rng(3)
    rows, width = 4, 1024
    hidden = rng.standard_normal((rows, width)).astype(np.float32)
    out = rng.standard_normal((rows, width)).astype(np.float32)
    gain = np.ones(width, np.float32)
    h = dev(hidden)
    normed = torch.zeros((rows, width), dtype=torch.float32, device="cuda")
    cb.run("norm", hidden=h, output=dev(out), gain=dev(gain), normed=normed, width=width, tokens=rows, add=1,
           last_token=1, epsilon=1e-6)
    done()
    same(h[:3].cpu().numpy(), hidden[:3])   # other rows untouched
    wh, wn = O.norm_row(hidden[3], out[3], gain, None, 1e-6, True)
    same(h[3].cpu().numpy(), wh)
    same(normed[3].cpu().numpy(), wn)


# ---- rope ----------------------------------------------------------------------

ROPE = [
    # name, d, Hq, Hkv, halves, qk_norm, base, factors
    ("qwen3", 128, 16, 8, True, True, 1e6, False),
    ("llama3", 64, 32, 8, False, False, 5e5, True),
    ("gemma3", 256, 4, 1, True, True, 1e4, False),
]


def llama3_factors(d, base):
    """The published llama3 rule (factor 32, low 1, high 4, original 8192)
    as a rope_freqs table; the reference only reads the tensor."""
    out = np.empty(d // 2, np.float32)
    factor, low, high, orig = 32.0, 1.0, 4.0, 8192.0
    for k in range(d // 2):
        freq = base ** (-2.0 * k / d)
        wavelen = 2 * math.pi / freq
        if wavelen < orig / high:
            out[k] = 1.0
        elif wavelen > orig / low:
            out[k] = factor
        else:
            smooth = (orig / wavelen - low) / (high - low)
            out[k] = 1.0 / ((1 - smooth) / factor + smooth)
    return out


@pytest.mark.parametrize("case", ROPE, ids=[c[0] for c in ROPE])
@pytest.mark.parametrize("position", [0, 5, 4097, 1 << 20])
def test_rope_bit_exact(cuda, case, position):
    name, d, hq, hkv, halves, qk, base, factors = case
    rng = np.random.default_rng(d + position % 97)
    tokens, slots = 3, 4608
    q = (rng.standard_normal((tokens, hq * d)) * 2).astype(np.float32)
    k = (rng.standard_normal((tokens, hkv * d)) * 2).astype(np.float32)
    v = rng.standard_normal((tokens, hkv * d)).astype(np.float32)
    qg = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32) if qk else None
    kg = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32) if qk else None
    turns = cb.rope_turns(base, d)
    fac = llama3_factors(d, base) if factors else None
    qd, kd, vd = dev(q), dev(k), dev(v)
    kc = torch.zeros((slots, hkv, d), dtype=torch.uint16, device="cuda")
    vc = torch.zeros((slots, hkv, d), dtype=torch.uint16, device="cuda")
    cb.run("rope", query=qd, key=kd, value=vd, key_cache=kc, value_cache=vc,
           query_gain=dev(qg) if qk else 0, key_gain=dev(kg) if qk else 0, factors=dev(fac) if factors else 0,
           turns=dev(turns), position=0, position0=position, tokens=tokens, head_dim=d, query_heads=hq,
           kv_heads=hkv, halves=int(halves), slots=slots, epsilon=1e-6)
    done()
    okc = np.zeros((slots, hkv, d), np.uint16)
    ovc = np.zeros((slots, hkv, d), np.uint16)
    for t in range(tokens):
        qt = q[t].copy()
        O.rope_token(qt, k[t], v[t], position + t, okc, ovc, head_dim=d, query_heads=hq, kv_heads=hkv,
                     halves=halves, slots=slots, epsilon=1e-6, turns=turns, factors=fac, query_gain=qg,
                     key_gain=kg)
        same(qd[t].cpu().numpy(), qt)
    same(kc.cpu().numpy(), okc)
    same(vc.cpu().numpy(), ovc)


# ---- attention -------------------------------------------------------------------

ATT = [
    # d, Hq, Hkv, window
    (128, 16, 8, 1 << 30),
    (64, 32, 8, 1 << 30),
    (256, 4, 1, 512),
    (256, 4, 1, 1 << 30),
]


def f16_cache(rng, slots, hkv, d, scale=1.0):
    return (rng.standard_normal((slots, hkv, d)) * scale).astype(np.float16).view(np.uint16)


@pytest.mark.parametrize("case", ATT, ids=[f"d{c[0]}_{c[1]}x{c[2]}_w{min(c[3], 9999)}" for c in ATT])
# steps of 32 rows or more take the many-query (prefill) kernel: same bits
@pytest.mark.parametrize("position,tokens", [(0, 1), (63, 1), (64, 1), (700, 1), (1000, 5), (40, 30),
                                             (0, 64), (40, 100), (500, 33), (1000, 130)])
def test_attention_bit_exact(cuda, case, position, tokens):
    d, hq, hkv, window = case
    rng = np.random.default_rng(position * 7 + tokens + d)
    slots = 2048
    kc = f16_cache(rng, slots, hkv, d, 2.0)
    vc = f16_cache(rng, slots, hkv, d)
    q = rng.standard_normal((tokens, hq * d)).astype(np.float32)
    scale_log2e = np.float32((1.0 / math.sqrt(d)) * 1.4426950408889634)
    max_chunks = (position + tokens + 63) // 64
    out = torch.zeros((tokens, hq * d), dtype=torch.float32, device="cuda")
    partials = torch.zeros(max_chunks * tokens * hq * d, dtype=torch.float32, device="cuda")
    stats = torch.zeros(max_chunks * tokens * hq * 2, dtype=torch.float32, device="cuda")
    tickets = torch.zeros(cb.lib().cb_attention_tickets(tokens, hq, hkv), dtype=torch.int32, device="cuda")
    cb.run("attention", query=dev(q), key_cache=dev(kc), value_cache=dev(vc), out=out, partials=partials,
           stats=stats, tickets=tickets, position=0, position0=position, tokens=tokens, head_dim=d, query_heads=hq,
           kv_heads=hkv, slots=slots, window=min(window, 0xFFFFFFFF), max_chunks=max_chunks,
           scale_log2e=float(scale_log2e))
    done()
    assert not tickets.any()   # left zero for the next step
    got = out.cpu().numpy()
    for t in range(tokens):
        p = position + t
        want = O.attention_row(q[t], p, kc, vc, slots, min(window, 0xFFFFFFFF), float(scale_log2e), d, hq, hkv)
        same(got[t], want)
        # tolerance against an f64 softmax
        kf = kc.view(np.float16).astype(np.float64)
        vf = vc.view(np.float16).astype(np.float64)
        early = p + 1 - window if p + 1 > window else 0
        for h in range(hq):
            g = h // (hq // hkv)
            keys = np.arange(early, p + 1)
            s = kf[keys % slots, g] @ q[t, h * d:(h + 1) * d].astype(np.float64) / math.sqrt(d)
            w = np.exp(s - s.max())
            ref = (w / w.sum()) @ vf[keys % slots, g]
            assert np.max(np.abs(got[t, h * d:(h + 1) * d] - ref)) <= 1e-4 * max(1.0, np.max(np.abs(ref)))


# ---- attention with the step's rope in its prologue --------------------------------

FUSED = [
    # name, d, Hq, Hkv, NEOX halves, QK-norm, base, llama3 factors, window
    ("qwen3", 128, 16, 8, True, True, 1e6, False, 1 << 30),
    ("llama3", 64, 32, 8, False, False, 5e5, True, 1 << 30),
    ("gemma3", 256, 4, 1, True, True, 1e4, False, 512),
]


@pytest.mark.parametrize("case", FUSED, ids=[c[0] for c in FUSED])
# 1500 with a full window: 24 live chunks, more than the 16 chunk CTAs (the
# newest key's chunk is then a later chunk of its CTA, copied from the cache)
@pytest.mark.parametrize("position", [0, 63, 64, 700, 1500])
@pytest.mark.parametrize("sequences", [0, 3])
def test_attention_fused_rope_matches_separate(cuda, case, position, sequences):
    """Decode attention with the step's rope folded into its prologue gives
    the bits of the rope launch followed by the attention launch: the
    outputs and both caches (the step's key and value appended)."""
    name, d, hq, hkv, halves, qk, base, factors, window = case
    rng = np.random.default_rng(position * 3 + sequences + d)
    rows, slots = max(sequences, 1), 2048
    stride = slots * hkv * d
    kc = f16_cache(rng, rows * slots, hkv, d, 2.0)
    vc = f16_cache(rng, rows * slots, hkv, d)
    q = (rng.standard_normal((rows, hq * d)) * 2).astype(np.float32)
    k = (rng.standard_normal((rows, hkv * d)) * 2).astype(np.float32)
    v = rng.standard_normal((rows, hkv * d)).astype(np.float32)
    qg = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32) if qk else None
    kg = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32) if qk else None
    turns = dev(cb.rope_turns(base, d))
    fac = dev(llama3_factors(d, base)) if factors else 0
    gains = dict(query_gain=dev(qg) if qk else 0, key_gain=dev(kg) if qk else 0)
    scale_log2e = float(np.float32((1.0 / math.sqrt(d)) * 1.4426950408889634))
    max_chunks = min(slots // 64, (position + 64) // 64 + 5)   # idle chunk CTAs too
    tickets_n = rows * hkv if sequences else cb.lib().cb_attention_tickets(1, hq, hkv)
    shape = dict(position=0, position0=position, tokens=rows, head_dim=d, query_heads=hq, kv_heads=hkv, slots=slots)
    seq = dict(rows_are_sequences=1, sequence_stride=stride) if sequences else {}
    outs = []
    for fused in (False, True):
        kcd, vcd, qd = dev(kc), dev(vc), dev(q)
        out = torch.zeros((rows, hq * d), dtype=torch.float32, device="cuda")
        partials = torch.zeros(max_chunks * rows * hq * d, dtype=torch.float32, device="cuda")
        stats = torch.zeros(max_chunks * rows * hq * 2, dtype=torch.float32, device="cuda")
        tickets = torch.zeros(tickets_n, dtype=torch.int32, device="cuda")
        rope = dict(query=qd, key=dev(k), value=dev(v), key_cache=kcd, value_cache=vcd, factors=fac, turns=turns,
                    halves=int(halves), epsilon=1e-6, **gains, **shape, **seq)
        if not fused:
            cb.run("rope", **rope)
        cb.run("attention", query=qd, key_cache=kcd, value_cache=vcd, out=out, partials=partials, stats=stats,
               tickets=tickets, window=min(window, 0xFFFFFFFF), max_chunks=max_chunks, scale_log2e=scale_log2e,
               rope=rope if fused else 0, **shape, **seq)
        done()
        assert not tickets.any()
        outs.append((out.cpu().numpy(), kcd.cpu().numpy(), vcd.cpu().numpy()))
    for a, b in zip(*outs):
        same(b, a)


# ---- gather ------------------------------------------------------------------------

@pytest.mark.parametrize("fmt,width,scale", [(O.Q6_K, 1024, 1.0), (O.Q4_0, 2048, 1.0),
                                             (O.Q8_0, 1152, float(np.sqrt(np.float32(1152)))),
                                             (O.Q8_0, 1024, 1.0), (O.Q4_1, 1024, 1.0),
                                             (O.BF16, 1152, float(np.sqrt(np.float32(1152))))])
def test_gather_bit_exact(cuda, fmt, width, scale):
    rng = np.random.default_rng(width + fmt)
    vocab = 300
    stored = synth.random_bytes_blocks(rng, fmt, vocab * width // O.BLOCK_WEIGHTS[fmt])
    piece = synth.to_piece(fmt, stored)
    nb = vocab * width // O.BLOCK_WEIGHTS[fmt]
    ids = np.array([5, 299, 0, 5, 123], np.uint32)
    hidden = torch.zeros((len(ids), width), dtype=torch.float32, device="cuda")
    cb.run("gather", piece=dev(piece), format=fmt, blocks=nb, width=width, first_row=0, row_count=vocab,
           ids=dev(ids), sampled=0, fed=0, tokens=len(ids), scale=scale, hidden=hidden)
    done()
    table = O.dequant_stored(fmt, stored).reshape(vocab, width)
    same(hidden.cpu().numpy(), (table[ids] * np.float32(scale)).astype(np.float32))


def test_gather_fed_reads_the_last_draw(cuda):
    rng = np.random.default_rng(2)
    vocab, width = 64, 256
    stored = synth.blocks(rng, O.Q6_K, vocab, width)
    nb = vocab * width // 256
    sampled = dev(np.array([17, 0, 0, 0], np.uint32))
    hidden = torch.zeros((1, width), dtype=torch.float32, device="cuda")
    cb.run("gather", piece=dev(synth.to_piece(O.Q6_K, stored)), format=O.Q6_K, blocks=nb, width=width, first_row=0,
           row_count=vocab, ids=0, sampled=sampled, fed=1, tokens=1, scale=1.0, hidden=hidden)
    done()
    same(hidden.cpu().numpy()[0], O.dequant_stored(O.Q6_K, stored).reshape(vocab, width)[17])


# ---- select and draw -------------------------------------------------------------------

def select(logits, **draw):
    count = logits.size
    tiles = cb.lib().cb_select_tiles(count)
    partials = torch.zeros(tiles * 128, dtype=torch.int32, device="cuda")
    ticket = torch.zeros(cb.lib().cb_select_tickets(count), dtype=torch.int32, device="cuda")
    cand = torch.zeros(128, dtype=torch.int32, device="cuda")
    rec = torch.zeros(4, dtype=torch.int32, device="cuda")
    min_p = draw.get("min_p", 0.0)
    cb.run("select", logits=dev(logits), count=count, partials=partials, ticket=ticket, candidates=cand, sampled=rec,
           position=0, position0=draw.get("position", 0), tokens=draw.get("tokens", 1), seed0=draw.get("seed0", 0),
           seed1=draw.get("seed1", 0), top_k=draw.get("top_k", 40), temperature=draw.get("temperature", 0.0),
           top_p=draw.get("top_p", 1.0), min_p=min_p, log_min_p=math.log(min_p) if min_p > 0 else 0.0)
    done()
    assert not ticket.any()
    return cand.cpu().numpy().view(np.uint32), rec.cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("count", [151936, 128256, 262144, 1024, 1000, 50])
def test_topk_matches_the_total_order(cuda, count):
    rng = np.random.default_rng(count)
    logits = (rng.standard_normal(count) * 3).astype(np.float32)
    # ties, signed zeros, a NaN, infinities (topk.wgsl:28-52)
    if count > 200:
        logits[10] = logits[20] = logits[30] = 9.0
        logits[40] = -0.0
        logits[41] = 0.0
        logits[count - 1] = np.inf
        logits[count - 2] = -np.inf
        logits[100] = np.nan
    cand, rec = select(logits)
    want = O.topk64(logits)
    same(cand, want)
    same(rec, O.draw(want, 0, 1))
    if count > 200:
        assert rec[1] == 1   # the top logit (NaN) is not finite: the draw fails


@pytest.mark.parametrize("settings", [dict(temperature=0.7, top_k=40, top_p=0.9, min_p=0.05, seed0=7, seed1=9),
                                      dict(temperature=1.0, top_k=64, top_p=1.0, seed0=1),
                                      dict(temperature=0.0, top_k=1)])
def test_draw_matches_oracle(cuda, settings):
    rng = np.random.default_rng(5)
    logits = rng.standard_normal(151936).astype(np.float32)
    cand, rec = select(logits, position=77, tokens=1, **settings)
    want = O.topk64(logits)
    same(cand, want)
    w = O.draw(want, 77, 1, seed=(settings.get("seed0", 0), settings.get("seed1", 0)),
               top_k=settings.get("top_k", 40), temperature=settings.get("temperature", 0.0),
               top_p=settings.get("top_p", 1.0), min_p=settings.get("min_p", 0.0))
    same(rec, w)
