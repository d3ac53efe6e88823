"""Host logic of the vocabulary split on CPU ranks (torch.distributed gloo,
world size 2): each rank's shard of a logit matrix, its top 64 with global
ids (the oracle's selection, topk.wgsl), the all-gather, and a merge under
the reference's total order must give every row the whole vocabulary's top
64. No GPU: this checks the partition, the id offsets and the list layout
the GPU merge reads ([world][rows][64] pairs)."""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from charlotte_b200.shard import shard_rows


def key_of(bits):
    b = np.uint32(bits)
    if b == 0x80000000:
        b = np.uint32(0)
    if (b & 0x7F800000) == 0x7F800000 and (b & 0x007FFFFF) != 0:
        return 0xFFFFFFFF
    return int(~b & 0xFFFFFFFF) if b & 0x80000000 else int(b | 0x80000000)


def merge(lists):
    """Top 64 of the union of (bits, id) lists: larger key first, lower id on ties."""
    pairs = [(int(b), int(i)) for lst in lists for b, i in lst.reshape(-1, 2) if i != 0xFFFFFFFF]
    pairs.sort(key=lambda p: (-key_of(p[0]), p[1]))
    out = np.full((64, 2), 0xFFFFFFFF, np.uint32)
    for j, (b, i) in enumerate(pairs[:64]):
        out[j] = (b, i)
    return out.reshape(-1)


def worker(rank, world, port, logits, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rows, vocab = logits.shape
    v0, v1 = shard_rows(vocab, world, rank)
    cand = np.empty((rows, 128), np.uint32)
    for r in range(rows):
        c = O.topk64(logits[r, v0:v1]).reshape(64, 2).copy()
        live = c[:, 1] != 0xFFFFFFFF
        c[live, 1] += v0
        cand[r] = c.reshape(-1)
    gathered = [torch.empty((rows, 128), dtype=torch.int64) for _ in range(world)]
    dist.all_gather(gathered, torch.from_numpy(cand.astype(np.int64)))
    lists = np.stack([g.numpy().astype(np.uint32) for g in gathered])   # [world][rows][128]
    ok = all(np.array_equal(merge(lists[:, r]), O.topk64(logits[r])) for r in range(rows))
    result[rank] = int(ok)
    dist.destroy_process_group()


def test_split_candidates_merge_to_whole_top64_gloo():
    rng = np.random.default_rng(3)
    logits = rng.standard_normal((5, 5000)).astype(np.float32)
    logits[0, 100:300] = 2.5          # ties across the shard boundary
    logits[1, :] = 0.0                # all equal: lowest ids win
    logits[2, 2499] = -0.0            # -0 equals +0
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    result = ctx.Array("i", 2)
    procs = [ctx.Process(target=worker, args=(r, 2, port, logits, result)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs)
    assert list(result) == [1, 1]


def test_shard_rows_cover_the_vocabulary():
    for vocab in (1000, 262144, 151936, 7):
        for world in (1, 2, 3, 8):
            spans = [shard_rows(vocab, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == vocab
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
