#!/usr/bin/env python3
"""Benchmark of the charlotte_b200 hot path on B200.

Headline (BASELINE.json metric "Q4_0/Q6_K GEMV HBM GB/s"): one step is one
pass of the decode GEMVs of a Qwen3-0.6B token over seeded random-init
weights (configs[1] at M = 1): 28 layers x [QKV 4096x1024, O 1024x2048,
gate|up 2x3072x1024, down 1024x3072] in Q4_0 and the 151,936x1024 Q6_K
head — 113 launches, 375.3 MB of weights a step (larger than the 126 MB L2,
so every step streams from HBM). The step is captured once as a CUDA graph
(PDL launches) and replayed. `value` = algorithmic bytes (weights + x + y)
/ time. `e2e` runs the same GEMVs through the C ABI with host buffers:
each step copies every x host->device and every y back inside the timed
region.

Beside the headline, the same JSON line carries every configuration of the
path, each with its roofline (and, at one GPU, a CPU baseline: the oracle
on the host cores): `qwen3_decode`, `gemma_batched_decode`
(configs[4], 64 sequences sharded over the ranks) and, at N > 1,
`gemma_split_head_decode` (the vocabulary-split head with its two NCCL
all-gathers a step, timed); at one GPU also `config1_q4_0_gemv`
(configs[0]), `sweep_m16_m128` (configs[1] at M = 16 and 128) and
`llama_prefill_decode`.

`--impl reference` times the reference path's CPU restatement (the oracle:
the reference's order of operations over its dequantizers, all host
threads) on a bounded sample of the same step.

Multi-GPU: the GEMV set does not shard (replicas only): each rank runs its
own replica, `value` is the sum over ranks, time the max over ranks.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from charlotte_b200 import synth  # noqa: E402

Q4_0, Q6_K = 2, 14
LAYERS, HIDDEN, FFN, VOCAB = 28, 1024, 3072, 151936
QKV_ROWS, ATT = 4096, 2048
SEED = 20261201
L2_BYTES = 126 * 1024 * 1024   # B200 L2


def qwen3_gemv_set():
    """(name, format, rows, K, members) of one decode token's products."""
    layer = [("qkv", Q4_0, [2048, 1024, 1024], HIDDEN), ("o", Q4_0, [HIDDEN], ATT),
             ("gate_up", Q4_0, [FFN, FFN], HIDDEN), ("down", Q4_0, [HIDDEN], FFN)]
    out = []
    for l in range(LAYERS):
        for name, fmt, rows, K in layer:
            out.append((f"{name}.{l}", fmt, rows, K))
    out.append(("head", Q6_K, [VOCAB], HIDDEN))
    return out


def algorithmic_bytes(fmt, rows_list, K):
    per_weight = 18 / 32 if fmt == Q4_0 else 210 / 256
    rows = sum(rows_list)
    out_rows = rows_list[0] if len(rows_list) == 2 else rows
    return rows * K * per_weight + 4 * K + 4 * out_rows


class Clocks:
    """nvidia-smi samples (every 200 ms) while the timed region runs."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(n_gpus):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(value, world):
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class GemvSet:
    """Device weights, inputs and outputs of one decode token's products."""

    def __init__(self, seed):
        import torch
        import charlotte_b200 as cb
        self.cb = cb
        rng = np.random.default_rng(seed)
        self.items = []
        self.bytes = 0.0
        spec = qwen3_gemv_set()
        # Every product's x in one contiguous buffer and every output in
        # another (16-byte aligned slices), so that the end-to-end run moves
        # a step's inputs and results with one copy each way.
        align = lambda n: (n + 3) // 4 * 4
        x_floats = sum(align(K) for _, _, _, K in spec)
        y_floats = sum(align(r) for _, _, rows, _ in spec for r in (rows if len(rows) != 2 else rows[:1]))
        self.xbuf = torch.empty(x_floats, dtype=torch.float32, device="cuda")
        self.ybuf = torch.zeros(y_floats, dtype=torch.float32, device="cuda")
        xo = yo = 0
        for name, fmt, rows, K in spec:
            members = []
            for r in rows:   # distinct weights for every layer and member
                stored = synth.blocks(rng, fmt, r, K)
                nb = stored.size // synth.BLOCK_BYTES[fmt]
                members.append((torch.from_numpy(synth.to_piece(fmt, stored)).cuda(), nb, 0, r, 0))
            kind = name.split(".")[0]
            epi = {"qkv": cb.QKV, "gate_up": cb.GATED}.get(kind, cb.WRITE)
            x = self.xbuf[xo: xo + K].view(1, K)
            x.copy_(torch.from_numpy(synth.activations(rng, 1, K)))
            xo += align(K)
            outs = []
            for r in (rows if epi == cb.QKV else rows[:1]):
                outs.append(self.ybuf[yo: yo + r].view(1, r))
                yo += align(r)
            self.items.append(dict(name=name, kind=kind, fmt=fmt, K=K, rows=rows, members=members, epi=epi, x=x,
                                   outs=outs, bytes=algorithmic_bytes(fmt, rows, K)))
            self.bytes += self.items[-1]["bytes"]

    def launch(self, item, stream, pdl=True):
        cb = self.cb
        cb.matmul(item["fmt"], item["K"], item["members"], item["x"], item["outs"], epilogue=item["epi"],
                  activation=cb.SILU, flags=cb.MATMUL_PDL if pdl else 0, stream=stream)

    def step(self, stream, events=None):
        for it in self.items:
            if events is not None and it["kind"] in events:
                ev = events[it["kind"]]
                ev[0].append(self._event(stream))
                self.launch(it, stream)
                ev[1].append(self._event(stream))
            else:
                self.launch(it, stream)

    @staticmethod
    def _event(stream):
        import torch
        e = torch.cuda.Event(enable_timing=True)
        e.record(stream)
        return e


def run_ours(args):
    import torch
    rank, world, local = dist_setup(args.gpus)
    import charlotte_b200 as cb
    cb.lib()
    gs = GemvSet(SEED + rank)
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    # warm-up (eager), then capture one step as a graph
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            gs.step(stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        gs.step(stream)
    torch.cuda.synchronize()
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()

    # Timed: K graph replays, CUDA events on the replay stream.
    clocks = Clocks(torch.cuda.current_device() if world == 1 else local)
    with clocks:
        time.sleep(0.3)
        barrier(world)
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        cur = torch.cuda.current_stream()
        start.record(cur)
        for _ in range(args.steps):
            graph.replay()
        end.record(cur)
        torch.cuda.synchronize()
        barrier(world)
        ms_total = start.elapsed_time(end)
        time.sleep(0.25)
    ms_total = max_over_ranks(ms_total, world)
    ms_per_step = ms_total / args.steps
    value = gs.bytes * world / (ms_per_step * 1e-3) / 1e9

    # Roofline of the dominant kernel: each kind of product (the 28 QKV, O,
    # gate|up, down launches; the head) captured alone as a CUDA graph of its
    # PDL launches and replayed, timed with CUDA events on the replay stream:
    # a launch's average duration inside a dependent chain, without the host.
    # The kind's weights are cloned until the graph reads more than twice L2
    # (28 QKV products alone are 66 MB), so every launch streams from HBM.
    per_kind, kind_bytes = {}, {}
    for kind in ("qkv", "o", "gate_up", "down", "head"):
        base = [it for it in gs.items if it["kind"] == kind]
        copies = max(1, int(np.ceil(2 * L2_BYTES / sum(it["bytes"] for it in base))))
        items = list(base)
        for _ in range(copies - 1):
            items += [dict(it, members=[(t.clone(), nb, f, r, o) for (t, nb, f, r, o) in it["members"]])
                      for it in base]
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for it in items:
                gs.launch(it, stream)
        reps = 20
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        cur = torch.cuda.current_stream()
        a.record(cur)
        for _ in range(reps):
            g.replay()
        b.record(cur)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / (reps * len(items))
        by = float(np.mean([it["bytes"] for it in items]))
        per_kind[kind] = dict(launches=len(items) * reps, ms=ms, gbs=by / (ms * 1e-3) / 1e9, copies=copies)
        kind_bytes[kind] = by * len(items) * reps
        del g, items
    q4_kinds = ("qkv", "o", "gate_up", "down")
    q4_ms = sum(per_kind[k]["ms"] * per_kind[k]["launches"] for k in q4_kinds)
    q4_launches = sum(per_kind[k]["launches"] for k in q4_kinds)
    q4_bytes = sum(kind_bytes[k] for k in q4_kinds)
    head = per_kind["head"]
    q4_step = sum(per_kind[k]["ms"] * len([it for it in gs.items if it["kind"] == k]) for k in q4_kinds)
    share_q4 = q4_step / (q4_step + head["ms"])
    peaks = read_peaks()
    dom = "decode_kernel<Q4_0>" if share_q4 >= 0.5 else "decode_kernel<Q6_K>"
    if share_q4 >= 0.5:
        achieved = (q4_bytes / q4_launches) / (q4_ms / q4_launches * 1e-3) / 1e9
        per_launch_bytes = q4_bytes / q4_launches
    else:
        achieved = head["gbs"]
        per_launch_bytes = gs.items[-1]["bytes"]
    peak = peaks.get("hbm_gbs", 6650.0)
    # DRAM traffic per launch: the ncu capture's DRAM bytes over the same
    # product's algorithmic bytes (profiles/gemv_q4_0_qkv_4096x1024.md:
    # 2,420,992 / 2,379,776; profiles/gemv_q6k_head_151936x1024.md:
    # 132,129,024 / 128,238,080), scaled to this launch's algorithmic bytes.
    traffic_ratio = 2420992 / 2379776 if share_q4 >= 0.5 else 132129024 / 128238080

    # e2e: the same products through the C ABI with host buffers.
    e2e = None if args.no_e2e else run_e2e(gs, graph, stream, max(args.steps // 4, 20), world)

    result = {
        "metric": "Q4_0/Q6_K GEMV HBM GB/s",
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32 (Q4_0/Q6_K weights)",
        "data": "synthetic: seeded random-init weights and N(0,1) activations",
        "config": {"workload": "qwen3-0.6b decode-token GEMV set (configs[1], M=1): 28x[QKV,O,gate|up,down] Q4_0 + head Q6_K",
                   "bytes_per_step": int(gs.bytes), "launches_per_step": len(gs.items),
                   "l2": "inputs larger than L2 (375 MB weights a step vs 126 MB L2)",
                   "parallelism": f"replicas x{world}", "graph": "CUDA graph of PDL launches"},
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "traffic": round(per_launch_bytes * traffic_ratio),
                     "traffic_source": "ncu DRAM bytes of the committed capture, scaled to this launch",
                     "bytes_per_launch": round(per_launch_bytes), "peak_source": "measured" if peaks else "fallback"},
        "per_product": {k: {kk: round(vv, 4) for kk, vv in v.items()} for k, v in per_kind.items()},
        "e2e": e2e,
        "gpu_launches": len(gs.items) * args.steps,
        "clocks": clocks.summary(),
    }
    cpu = not args.no_cpu_baseline
    if not args.no_decode:
        result["qwen3_decode"] = decode_bench(args.decode_steps, 512, SEED + 7 + rank, world)
    if not args.no_batch:
        result["gemma_batched_decode"] = gemma_batch_bench(args.batch_steps, world, rank, cpu=cpu)
        if world > 1:
            # the vocabulary-split head (the path's one exchange) beside the sequence-sharded run
            result["gemma_split_head_decode"] = gemma_split_bench(args.batch_steps, world, rank)
    if world == 1 and not args.no_configs:
        # the single-GPU configurations: configs[0], configs[1] at M = 16 and 128, configs[3]
        result["config1_q4_0_gemv"] = config1_bench(cpu=cpu)
        result["sweep_m16_m128"] = sweep_summary(sweep_bench(iters=20, ms=[16, 128], formats=(2,), head=True))
        result["llama_prefill_decode"] = llama_bench(128, SEED + 11, cpu=cpu)
    if rank == 0 and world == 1 and cpu:
        result["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
        if "qwen3_decode" in result:
            result["qwen3_decode"]["cpu_baseline"] = cpu_decode_baseline(SEED + 7)
    if rank == 0:
        print(json.dumps(result), flush=True)
    del graph
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_e2e(gs, graph, stream, steps, world):
    """The same products end to end with host buffers: each step copies every
    product's x from one pinned host buffer to the device (one copy), replays
    the captured graph of C ABI launches, and copies every output back to one
    pinned host buffer (one copy); all three inside the timed region, on the
    replay stream."""
    import torch
    hx = gs.xbuf.cpu().pin_memory()
    hy = torch.empty_like(gs.ybuf, device="cpu").pin_memory()
    h2d = hx.numel() * 4
    d2h = hy.numel() * 4

    def one():
        with torch.cuda.stream(stream):
            gs.xbuf.copy_(hx, non_blocking=True)
            graph.replay()
            hy.copy_(gs.ybuf, non_blocking=True)
    for _ in range(3):
        one()
    torch.cuda.synchronize()
    barrier(world)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        one()
    end.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(start.elapsed_time(end), world) / steps
    return {"value": round(gs.bytes * world / (ms * 1e-3) / 1e9, 1), "unit": "GB/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(ms, 4),
            "how": "one pinned host->device copy of every x, the captured graph of cb_matmul_run launches, one "
                   "device->host copy of every output, a step"}


def decode_bench(steps, prompt_len, seed, world):
    """Qwen3-0.6B greedy decode, a 512-token prompt then `steps`
    fed decode steps (one CUDA graph replayed), random-init weights."""
    import torch
    from charlotte_b200 import model as M
    arch = M.qwen3_0_6b(context=4096)
    m = M.synthesize(arch, seed=seed)
    dec = M.Decoder(m, max_step_tokens=512)
    rng = np.random.default_rng(seed + 1)
    prompt = rng.integers(0, arch.vocab, prompt_len).astype(np.uint32)
    t0 = time.perf_counter()
    rec = dec.prefill(prompt)
    prefill_s = time.perf_counter() - t0
    dec.generate(4)   # capture and warm the decode graph
    # restart from the prompt so the timed run is the configured one (warm)
    t0 = time.perf_counter()
    rec = dec.prefill(prompt)
    prefill_warm_s = time.perf_counter() - t0
    barrier(world)
    toks, failed, dev_ms = dec.generate(steps, timed=True)
    dev_ms = max_over_ranks(dev_ms, world)
    # e2e: the same steps driven from the host one at a time through
    # cb_decoder_step (each step: the token id host->device, the 16-byte
    # record device->host), after the same prompt.
    rec = dec.prefill(prompt)
    tok = int(rec[0])
    barrier(world)
    t0 = time.perf_counter()
    host_toks = []
    for i in range(steps):
        r = dec.step(np.array([tok], np.uint32), prompt_len + i)
        tok = int(r[0])
        host_toks.append(tok)
    e2e_s = max_over_ranks(time.perf_counter() - t0, world)
    dec.close()
    return {
        "workload": "qwen3-0.6b greedy decode (configs[2]): 512-token prompt, %d steps, f16 KV, context 4096" % steps,
        "tok_s": round(steps * world / (dev_ms * 1e-3), 1),
        "ms_per_token": round(dev_ms / steps, 4),
        "roofline": decode_roofline(m, range(prompt_len, prompt_len + steps), dev_ms / steps),
        # gather, then a layer's QKV (its norm folded in), attention (its rope
        # folded in), O, gate|up (norm folded in), down; the head (final norm
        # folded in), top-k + draw, the position advance
        "launches_per_token": 4 + 5 * arch.layers,
        "prefill_512_ms_wall": round(prefill_warm_s * 1e3, 1),
        "prefill_512_ms_wall_first": round(prefill_s * 1e3, 1),
        "host_driven_matches_graph": bool(host_toks == toks.tolist()),
        "failed_steps": int(failed.sum()),
        "e2e": {"value": round(steps * world / e2e_s, 1), "unit": "tok/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 16, "how": "cb_decoder_step per token from host ids, record read back"},
    }


def llama_bench(decode_steps, seed, cpu=True, forms=(True, False), profile=False):
    """Llama-3.2-1B shapes, random-init weights, a 2,048-token
    prompt as four 512-token steps on the tcgen05 path
    (CB_DECODER_TENSOR_PREFILL), then `decode_steps` greedy decode steps
    (exact form, one CUDA graph replayed). The same prompt through the exact
    forms is timed beside it. Prefill is wall-timed around the four
    synchronous steps (host calls included); its roofline is the tensor
    form's FLOPs (every layer product, the causal attention, the last
    token's head) over that time against the measured sustained bf16 tensor
    peak; decode's is bytes a token against HBM."""
    import torch
    from charlotte_b200 import model as M
    arch = M.llama_3_2_1b(context=2048 + decode_steps + 64)
    m = M.synthesize(arch, seed=seed)
    rng = np.random.default_rng(seed + 1)
    P = 2048
    prompt = rng.integers(0, arch.vocab, P).astype(np.uint32)
    out = {"workload": "llama-3.2-1b shapes (configs[3]): 2048-token prompt as 4x512 steps, "
                       "then %d greedy steps" % decode_steps}
    layer_params = sum(w.rows * w.cols for L in m.layers for w in (L.q, L.k, L.v, L.o, L.gate, L.up, L.down))
    head = m.output if m.output is not None else m.token_embd
    attention_flops = 4.0 * arch.head_dim * arch.query_heads * arch.layers * (P * (P + 1) / 2)
    flops = 2.0 * P * layer_params + attention_flops + 2.0 * head.rows * head.cols
    peaks = read_peaks()
    tensor_peak = peaks.get("bf16_tflops_sustained", 1370.0)
    for tensor in forms:
        dec = M.Decoder(m, max_step_tokens=512, tensor_prefill=tensor)
        dec.prefill(prompt)   # warm
        if profile:
            profiled_region(lambda: dec.prefill(prompt))
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        rec = dec.prefill(prompt)
        sec = time.perf_counter() - t0
        key = "prefill_tensor" if tensor else "prefill_exact"
        tflops = flops / sec / 1e12
        out[key] = {"ms": round(sec * 1e3, 2), "tok_s": round(P / sec, 1), "tflops": round(tflops, 1),
                    "flops": flops}
        if tensor:
            out[key]["roofline"] = {"bound": "tensor", "kernel": "prefill step (all launches)",
                                    "achieved": round(tflops, 1), "peak": tensor_peak, "unit": "TFLOP/s",
                                    "frac": round(tflops / tensor_peak, 4), "traffic": None,
                                    "peak_source": "measured sustained" if peaks else "fallback"}
            dec.generate(4)
            dec.prefill(prompt)
            toks, failed, dev_ms = dec.generate(decode_steps, timed=True)
            out["decode"] = {"tok_s": round(decode_steps / (dev_ms * 1e-3), 1),
                             "ms_per_token": round(dev_ms / decode_steps, 4), "failed_steps": int(failed.sum()),
                             "roofline": decode_roofline(m, range(P, P + decode_steps), dev_ms / decode_steps)}
        else:
            out[key]["note"] = "exact f32 forms on the CUDA cores (the reference's order of operations)"
        dec.close()
    if cpu:
        out["cpu_baseline"] = cpu_model_decode_baseline(M.llama_3_2_1b(context=64), seed)
    return out


def profiled_region(fn):
    """Runs fn() between cudaProfilerStart and cudaProfilerStop: the one
    region an `ncu --profile-from-start off` launch list captures."""
    import torch
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    try:
        return fn()
    finally:
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()


def gemma_batch_bench(steps, world, rank, sequences=64, prompt_len=1024, cpu=True, profile=False):
    """Gemma-3-1B shapes, random-init weights; 64 independent
    sequences with random 1,024-token prompts, sharded over the ranks (64/N
    each, no collective on the data path: strong scaling of a fixed batch);
    each rank prefills its sequences, then all step together, one token per
    sequence a step, as one replayed CUDA graph. tok/s = all sequences'
    tokens / the max over ranks of the device time."""
    from charlotte_b200 import model as M
    assert sequences % world == 0
    S = sequences // world
    arch = M.gemma_3_1b(context=prompt_len + steps + 64)
    m = M.synthesize(arch, seed=SEED + 21)   # the same weights on every rank
    bd = M.BatchDecoder(m, S, max_step_tokens=512)
    for s in range(S):
        g = rank * S + s   # global sequence id
        prompt = np.random.default_rng(SEED + 1000 + g).integers(0, arch.vocab, prompt_len).astype(np.uint32)
        bd.prefill_sequence(s, prompt)
    bd.generate(3)   # capture and warm the batched graph
    for s in range(S):   # restart every sequence from its prompt
        g = rank * S + s
        prompt = np.random.default_rng(SEED + 1000 + g).integers(0, arch.vocab, prompt_len).astype(np.uint32)
        bd.prefill_sequence(s, prompt)
    barrier(world)
    toks, failed, dev_ms = bd.generate(steps, timed=True)
    dev_local = dev_ms
    dev_ms = max_over_ranks(dev_ms, world)
    if profile:
        profiled_region(lambda: bd.generate(1))
    bd.close()
    out = {"workload": "gemma-3-1b shapes (configs[4]): %d sequences x %d-token prompts, %d batched steps" % (
                sequences, prompt_len, steps),
           "sequences_per_gpu": S, "tok_s": round(sequences * steps / (dev_ms * 1e-3), 1),
           "ms_per_step": round(dev_ms / steps, 4), "scaling": "strong (64 sequences in all, split over ranks)",
           "failed_steps": int(failed.sum()),
           # one rank's step: its sequences' KV reads and the whole weights
           "roofline": decode_roofline(m, range(prompt_len, prompt_len + steps), dev_local / steps, rows=S,
                                       kernel="batched decode step on one rank (all launches)"),
           "head": "tied Q8_0 262,144 x 1,152 (Q6_K needs widths of whole 256-weight super-blocks)"}
    if rank == 0 and world == 1 and cpu:
        out["cpu_baseline"] = cpu_model_decode_baseline(M.gemma_3_1b(context=64), SEED + 21, steps=3)
        out["cpu_baseline"]["sample"] += " (one sequence: the GPU figure steps 64)"
    return out


def gemma_split_bench(steps, world, rank, sequences=64, prompt_len=1024):
    """configs[4] with the head split by vocabulary: sequences sharded as in
    gemma_batch_bench for the layers; per step the normed rows are
    all-gathered (NCCL), each rank computes its vocabulary shard of the head
    for all 64 rows and its top 64 (global ids), the candidate lists are
    all-gathered, and every rank merges and draws (charlotte_b200.shard).
    Timed with CUDA events on the decoder's stream around the steps (host
    orchestration between launches included)."""
    import torch
    from charlotte_b200 import model as M
    from charlotte_b200 import shard
    assert sequences % world == 0
    S = sequences // world
    arch = M.gemma_3_1b(context=prompt_len + steps + 64)
    m = M.synthesize(arch, seed=SEED + 21)
    bd = M.BatchDecoder(m, S, max_step_tokens=512)

    def prefill():
        for s in range(S):
            g = rank * S + s
            prompt = np.random.default_rng(SEED + 1000 + g).integers(0, arch.vocab, prompt_len).astype(np.uint32)
            bd.prefill_sequence(s, prompt)
    sh = shard.SplitHead(bd, sequences, world, rank)
    prefill()
    for i in range(3):   # warm
        sh.step(prompt_len + i)
    prefill()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(sh.stream)
    toks = []
    timing = []
    for i in range(steps):
        sh.step(prompt_len + i, timing=timing)
        toks.append(sh.sampled_all[:, 0])
    e1.record(sh.stream)
    torch.cuda.synchronize()
    dev_ms = max_over_ranks(e0.elapsed_time(e1), world)
    gather_ms = max_over_ranks(sum(a.elapsed_time(b) + c.elapsed_time(d) for a, b, c, d in timing) / steps, world)
    bd.close()
    return {"workload": "gemma-3-1b shapes (configs[4]) with a vocabulary-split head: %d sequences x %d-token "
                        "prompts, %d steps" % (sequences, prompt_len, steps),
            "sequences_per_gpu": S, "vocab_rows_per_gpu": arch.vocab // world,
            "tok_s": round(sequences * steps / (dev_ms * 1e-3), 1), "ms_per_step": round(dev_ms / steps, 4),
            "allgather_ms_per_step": round(gather_ms, 4),
            "collectives_per_step": "all-gather of normed rows (%d B) + all-gather of candidates (%d B) a rank" % (
                S * arch.hidden * 4, sequences * 128 * 4)}


def config1_bench(iters=200, cpu=True):
    """one Q4_0 GEMV, W [8192, 2048] (Llama-3.2-1B gate_proj),
    d = |N(0,0.02)|/8, x ~ N(0,1): GB/s graph-timed over copies of W that
    together exceed L2, the bits checked against the oracle, and the oracle
    timed on the host cores for the same product."""
    import torch
    import charlotte_b200 as cb
    import oracle as O
    torch.cuda.set_device(0)
    rng = np.random.default_rng(SEED + 1)
    rows, K = 8192, 2048
    stored = synth.blocks(rng, Q4_0, rows, K)
    nb = stored.size // synth.BLOCK_BYTES[Q4_0]
    piece_h = synth.to_piece(Q4_0, stored)
    piece = torch.from_numpy(piece_h).cuda()
    copies = int(np.ceil(256e6 / piece.numel()))
    pieces = [piece] + [piece.clone() for _ in range(copies - 1)]
    xh = synth.activations(rng, 1, K)
    x = torch.from_numpy(xh).cuda()
    y = torch.empty((1, rows), dtype=torch.float32, device="cuda")

    def launch(i):
        cb.matmul(Q4_0, K, [(pieces[i % copies], nb, 0, rows, 0)], x, [y], flags=cb.MATMUL_PDL)
    ms = graph_time_ms(launch, iters)
    cb.matmul(Q4_0, K, [(piece, nb, 0, rows, 0)], x, [y])
    torch.cuda.synchronize()
    exact = bool(np.array_equal(y.cpu().numpy(), O.matmul(Q4_0, piece_h, nb, rows, K, xh)))
    nbytes = rows * K * 18 / 32 + 4 * K + 4 * rows
    peaks = read_peaks()
    peak = peaks.get("hbm_gbs", 6650.0)
    gbs = nbytes / (ms * 1e-3) / 1e9
    out = {"workload": "configs[0]: Q4_0 GEMV 8192 x 2048", "us": round(ms * 1e3, 2), "gbs": round(gbs, 1),
           "bit_exact_vs_oracle": exact,
           "roofline": {"bound": "hbm", "kernel": "decode_kernel<Q4_0>", "achieved": round(gbs, 1), "peak": peak,
                        "unit": "GB/s", "frac": round(gbs / peak, 4), "traffic": None,
                        "bytes_per_launch": round(nbytes), "peak_source": "measured" if peaks else "fallback",
                        "how": "%d launches in a CUDA graph over copies of W totalling more than L2" % iters}}
    if cpu:
        threads = os.cpu_count() or 1
        O.matmul(Q4_0, piece_h, nb, rows, K, xh, threads=threads)
        t0 = time.perf_counter()
        n = 0
        while time.perf_counter() - t0 < 3.0:
            O.matmul(Q4_0, piece_h, nb, rows, K, xh, threads=threads)
            n += 1
        cpu_s = (time.perf_counter() - t0) / n
        out["cpu_baseline"] = {"value": round(nbytes / cpu_s / 1e9, 2), "unit": "GB/s", "cores": threads,
                               "kind": "port", "sample": "%d runs of the same product, oracle, %.1f s" % (
                                   n, time.perf_counter() - t0)}
    return out


def cpu_decode_baseline(seed):
    """The oracle's pass (the reference's order of operations) on all host
    cores: a 16-token prompt then 4 decode steps of Qwen3-0.6B."""
    from charlotte_b200 import model as M
    from oracle.model import OracleDecoder
    m = M.synthesize(M.qwen3_0_6b(context=64), seed=seed)
    od = OracleDecoder(m)
    rng = np.random.default_rng(seed + 1)
    rec, _ = od.step(rng.integers(0, 151936, 16).astype(np.uint32), 0, logits=False)
    rec, _ = od.step([1], 16)
    t0 = time.perf_counter()
    n = 4
    tok = rec[0]
    for i in range(n):
        rec, _ = od.step([tok], 17 + i)
        tok = rec[0]
    el = time.perf_counter() - t0
    od.close()
    return {"value": round(n / el, 2), "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"Qwen3-0.6B decode, 4 steps after 17 positions, oracle, {os.cpu_count()} threads, {el:.1f} s"}


def read_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return {}


BYTES_PER_WEIGHT_ALL = {2: 18 / 32, 3: 20 / 32, 8: 34 / 32, 14: 210 / 256, 30: 2.0}


def weight_bytes(model):
    """Algorithmic bytes of a decode token's weights: every layer product and
    the head (the table itself when tied), each read once."""
    layers = sum(w.rows * w.cols * BYTES_PER_WEIGHT_ALL[w.format] for L in model.layers
                 for w in (L.q, L.k, L.v, L.o, L.gate, L.up, L.down))
    head = model.output if model.output is not None else model.token_embd
    return layers, head.rows * head.cols * BYTES_PER_WEIGHT_ALL[head.format]


def kv_read_bytes(arch, position):
    """f16 keys and values attention reads for one query at `position`:
    every layer's live keys (its window, or position + 1)."""
    per_key = 2 * arch.kv_heads * arch.head_dim * 2
    return sum(min(arch.layer_window(l), position + 1) for l in range(arch.layers)) * per_key


def decode_roofline(model, positions, ms_per_step, rows=1, kernel="decode step (all launches)"):
    """A decode step's algorithmic bytes (the weights once, each row's KV
    reads at the steps' mean position) over its measured time, against the
    measured HBM peak."""
    layers, head = weight_bytes(model)
    kv = rows * float(np.mean([kv_read_bytes(model.arch, p) for p in positions]))
    nbytes = layers + head + kv
    peak = read_peaks().get("hbm_gbs")
    achieved = nbytes / (ms_per_step * 1e-3) / 1e9
    return {"bound": "hbm", "kernel": kernel, "achieved": round(achieved, 1), "peak": peak or 6650.0,
            "unit": "GB/s", "frac": round(achieved / (peak or 6650.0), 4), "traffic": None,
            "bytes_per_step": round(nbytes), "weight_bytes": round(layers + head), "kv_bytes": round(kv),
            "peak_source": "measured" if peak else "fallback"}


def cpu_model_decode_baseline(arch, seed, prompt=16, steps=4, threads=0):
    """The oracle's pass (the reference's order of operations) on the host
    cores: a short prompt, then `steps` greedy decode steps of one sequence."""
    from charlotte_b200 import model as M
    from oracle.model import OracleDecoder
    m = M.synthesize(arch, seed=seed)
    od = OracleDecoder(m, threads=threads)
    rng = np.random.default_rng(seed + 1)
    rec, _ = od.step(rng.integers(0, arch.vocab, prompt).astype(np.uint32), 0, logits=False)
    rec, _ = od.step([1], prompt)
    tok = rec[0]
    t0 = time.perf_counter()
    for i in range(steps):
        rec, _ = od.step([tok], prompt + 1 + i)
        tok = rec[0]
    el = time.perf_counter() - t0
    od.close()
    return {"value": round(steps / el, 2), "unit": "tok/s", "cores": od.threads, "kind": "port",
            "sample": f"{arch.name} decode of one sequence, {steps} steps after {prompt + 1} positions, oracle, "
                      f"{od.threads} threads, {el:.1f} s"}


def cpu_sample_items(fraction=1.0):
    """A bounded sample of the step for the CPU: one layer's four products
    and 1/16 of the head's rows, each cut to `fraction` of its rows."""
    f = lambda r: max(32, int(r * fraction) // 32 * 32)
    return [("qkv", Q4_0, [f(2048), f(1024), f(1024)], HIDDEN), ("o", Q4_0, [f(HIDDEN)], ATT),
            ("gate_up", Q4_0, [f(FFN), f(FFN)], HIDDEN), ("down", Q4_0, [f(HIDDEN)], FFN),
            ("head/16", Q6_K, [f(VOCAB // 16)], HIDDEN)]


def cpu_baseline(seconds, repeat=None, fraction=1.0):
    import oracle as O
    rng = np.random.default_rng(SEED)
    prepared = []
    total_bytes = 0.0
    for name, fmt, rows_list, K in cpu_sample_items(fraction):
        for rows in rows_list:
            stored = synth.blocks(rng, fmt, rows, K)
            nb = stored.size // synth.BLOCK_BYTES[fmt]
            prepared.append((fmt, O.to_piece(fmt, stored), nb, rows, K, synth.activations(rng, 1, K)))
        total_bytes += algorithmic_bytes(fmt, rows_list, K)
    threads = os.cpu_count() or 1
    O.lib()
    t0 = time.perf_counter()
    n = 0
    while True:
        for fmt, piece, nb, rows, K, x in prepared:
            O.matmul(fmt, piece, nb, rows, K, x, threads=threads)
        n += 1
        el = time.perf_counter() - t0
        if (repeat is not None and n >= repeat) or (repeat is None and el >= seconds):
            break
    gbs = total_bytes * n / el / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "seconds": el,
            "sample": f"{fraction:g} of one Qwen3 layer's 4 Q4_0 products + 1/16 of the Q6_K head "
                      f"({total_bytes / 1e6:.2f} MB) x{n}, {el:.1f} s, oracle (reference order of operations), "
                      f"{threads} threads"}


def run_reference(args):
    """The reference path's CPU restatement on the host cores, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    # Size each step so that the whole run stays near a minute of CPU time:
    # the full sample takes ~0.12 s on 8 cores.
    probe = cpu_baseline(0, repeat=1)
    fraction = min(1.0, max(1.0 / 64, 45.0 / (max(args.steps + args.warmup, 1) * max(probe["seconds"], 1e-3))))
    for _ in range(args.warmup):
        cpu_baseline(0, repeat=1, fraction=fraction)
    t0 = time.perf_counter()
    vals = [cpu_baseline(0, repeat=1, fraction=fraction) for _ in range(args.steps)]
    el = time.perf_counter() - t0
    value = float(np.median([v["value"] for v in vals]))
    line = {
        "impl": "reference",
        "metric": "Q4_0/Q6_K GEMV HBM GB/s",
        "value": round(value, 3),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(el / max(args.steps, 1) * 1e3, 2),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32 (Q4_0/Q6_K weights)",
        "data": "synthetic: seeded random-init weights and N(0,1) activations",
        "config": {"workload": "qwen3-0.6b decode-token GEMV set (configs[1], M=1): 28x[QKV,O,gate|up,down] Q4_0 + head Q6_K",
                   "sample": "each step: one layer's 4 products + 1/16 of the head"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
                         "sample": vals[0]["sample"]},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_case(spec, iters):
    """One product launched `iters` times (for profiling): spec is
    format:rows:K[:tokens[:form]], form one of tensor, dense (the tensor form
    over weights densified first), split, tiled, streamed, e.g.
    q4_0:1024:2048, q4_0:4096:1024:512, q4_0:4096:1024:2048:tensor or
    q4_0:1152:6912:64:split. Prints the mean device time a launch."""
    import torch
    import charlotte_b200 as cb
    fmt_name, rows, K, *rest = spec.split(":")
    fmt = {"q4_0": Q4_0, "q6_k": Q6_K, "q8_0": 8}[fmt_name]
    rows, K = int(rows), int(K)
    tokens = int(rest[0]) if rest else 1
    form = rest[1] if len(rest) > 1 else ""
    flags = {"tensor": cb.MATMUL_TENSOR, "dense": cb.MATMUL_TENSOR, "split": cb.MATMUL_SPLIT,
             "tiled": cb.MATMUL_TILED, "streamed": cb.MATMUL_STREAMED}.get(form, 0)
    scratch = None
    if form == "split":
        scratch = torch.empty(cb.lib().cb_matmul_split_bytes(tokens, rows) // 4, dtype=torch.float32, device="cuda")
    if form == "dense":
        n = cb.lib().cb_matmul_scratch_bytes(flags, tokens, K) + 8 * tokens * rows * 4
        scratch = torch.empty(n, dtype=torch.uint8, device="cuda")
    torch.cuda.set_device(0)
    rng = np.random.default_rng(SEED)
    stored = synth.blocks(rng, fmt, rows, K)
    nb = stored.size // synth.BLOCK_BYTES[fmt]
    piece = torch.from_numpy(synth.to_piece(fmt, stored)).cuda()
    members = [(piece, nb, 0, rows, 0)]
    dense = cb.densify(fmt, K, members) if form == "dense" else None
    x = torch.from_numpy(synth.activations(rng, tokens, K)).cuda()
    y = torch.zeros((tokens, rows), dtype=torch.float32, device="cuda")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for i in range(iters):
        if i == 1:
            e0.record()
        cb.matmul(fmt, K, members, x, [y], flags=flags | cb.MATMUL_PDL, scratch=scratch, dense=dense)
    e1.record()
    torch.cuda.synchronize()
    cb.check(cb.lib().cb_fault_check(None))
    us = e0.elapsed_time(e1) * 1e3 / max(iters - 1, 1)
    print(json.dumps({"case": spec, "iters": iters, "ok": True, "us": round(us, 2),
                      "tflops": round(2.0 * tokens * rows * K / us / 1e6, 1)}))


SWEEP_SHAPES = [("qkv", 4096, 1024), ("o", 1024, 2048), ("gate_up", 6144, 1024), ("down", 1024, 3072)]
SWEEP_M = [1, 16, 128, 512, 2048]
BYTES_PER_WEIGHT = {2: 18 / 32, 8: 34 / 32, 14: 210 / 256}
FORMAT_NAME = {2: "Q4_0", 8: "Q8_0", 14: "Q6_K"}


def graph_time_ms(launch, n):
    """Mean device ms of `launch(i)` for i in range(n), captured once as a CUDA
    graph (no host launch cost in the timing) and replayed after a warm
    replay, timed with CUDA events on the replay stream."""
    import torch
    launch(0)   # first calls outside capture (kernel attributes)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(n):
            launch(i)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) / n


def sweep_bench(iters=20, flags=0, ms=None, formats=(8, 2, 14), head=True):
    """the Qwen3-shape product sweep. Each (format, shape, M):
    `iters` launches in a CUDA graph, weights rotated over copies totalling
    more than 2x L2 so that every launch reads them from HBM. Reports GB/s
    (weights + x + y) and TFLOP/s (2MNK)."""
    import torch
    import charlotte_b200 as cb
    torch.cuda.set_device(0)
    rng = np.random.default_rng(SEED + 3)
    cases = [(fmt, name, rows, K) for fmt in formats for name, rows, K in SWEEP_SHAPES]
    if head:
        cases.append((14, "head", VOCAB, HIDDEN))
    rows_out = []
    for fmt, name, rows, K in cases:
        stored = synth.blocks(rng, fmt, rows, K)
        nb = stored.size // synth.BLOCK_BYTES[fmt]
        piece = torch.from_numpy(synth.to_piece(fmt, stored)).cuda()
        copies = max(1, min(64, int(np.ceil(256e6 / piece.numel()))))
        pieces = [piece] + [piece.clone() for _ in range(copies - 1)]
        for M in (ms or SWEEP_M):
            x = torch.from_numpy(synth.activations(rng, M, K)).cuda()
            y = torch.empty((M, rows), dtype=torch.float32, device="cuda")
            n = iters if M * rows < 2048 * 8192 else 4

            def launch(i):
                cb.matmul(fmt, K, [(pieces[i % copies], nb, 0, rows, 0)], x, [y], flags=flags)
            t = graph_time_ms(launch, n)
            cb.check(cb.lib().cb_fault_check(None))
            nbytes = rows * K * BYTES_PER_WEIGHT[fmt] + 4 * M * (K + rows)
            rows_out.append({"format": FORMAT_NAME[fmt], "product": name, "N": rows, "K": K, "M": M,
                             "us": round(t * 1e3, 2), "gbs": round(nbytes / t / 1e6, 1),
                             "tflops": round(2 * M * rows * K / t / 1e9, 2)})
            del x, y
        del pieces, piece
        torch.cuda.empty_cache()
    form = ("tensor" if flags & 2 else "streamed" if flags & 4 else "tiled" if flags & 8 else
            "exact, form chosen by size")
    return {"workload": "configs[1]: Qwen3-shape product sweep", "form": form, "results": rows_out}


def split_forms_bench(iters=10):
    """The split form beside the streamed and tiled exact forms on the
    few-tile, wide-K products it is for (Qwen3's O and down, Llama's O and
    down, Gemma's down), at the token counts a batched decode or a prefill
    step gives them: device µs a launch, weights rotated over copies larger
    than L2."""
    import torch
    import charlotte_b200 as cb
    torch.cuda.set_device(0)
    rng = np.random.default_rng(SEED + 5)
    shapes = [("qwen3.o", 1024, 2048), ("qwen3.down", 1024, 3072), ("llama.o", 2048, 2048),
              ("llama.down", 2048, 8192), ("gemma.down", 1152, 6912)]
    rows_out = []
    for name, rows, K in shapes:
        stored = synth.blocks(rng, Q4_0, rows, K)
        nb = stored.size // synth.BLOCK_BYTES[Q4_0]
        piece = torch.from_numpy(synth.to_piece(Q4_0, stored)).cuda()
        copies = max(1, min(16, int(np.ceil(256e6 / piece.numel()))))
        pieces = [piece] + [piece.clone() for _ in range(copies - 1)]
        for M in (4, 8, 16, 32, 64, 128, 256, 512):
            x = torch.from_numpy(synth.activations(rng, M, K)).cuda()
            y = torch.empty((M, rows), dtype=torch.float32, device="cuda")
            rs = torch.empty(cb.lib().cb_matmul_split_bytes(M, rows) // 4, dtype=torch.float32, device="cuda")
            row = {"product": name, "N": rows, "K": K, "M": M}
            for form, flags, scratch in (("streamed", cb.MATMUL_STREAMED, None), ("tiled", cb.MATMUL_TILED, None),
                                         ("split", cb.MATMUL_SPLIT, rs), ("auto", 0, rs)):
                def launch(i, flags=flags, scratch=scratch):
                    cb.matmul(Q4_0, K, [(pieces[i % copies], nb, 0, rows, 0)], x, [y], flags=flags | cb.MATMUL_PDL,
                              scratch=scratch)
                row[form] = round(graph_time_ms(launch, iters) * 1e3, 2)
            cb.check(cb.lib().cb_fault_check(None))
            rows_out.append(row)
    return {"workload": "split form vs the exact forms, Q4_0", "unit": "us a launch", "results": rows_out}


def sweep_summary(sweep):
    """The sweep's rows with each one's roofline fraction: HBM for M = 16
    (weights dominate the bytes), the sustained tensor peak for the others
    (their exact forms run on the CUDA cores, so the fraction says how far
    the exact order is from the tensor cores)."""
    peaks = read_peaks()
    hbm = peaks.get("hbm_gbs", 6650.0)
    tensor = peaks.get("bf16_tflops_sustained", 1370.0)
    for r in sweep["results"]:
        r["frac_hbm"] = round(r["gbs"] / hbm, 4)
        r["frac_tensor_sustained"] = round(r["tflops"] / tensor, 4)
    sweep["peak_source"] = "measured" if peaks else "fallback"
    return sweep


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--decode-steps", type=int, default=256)
    ap.add_argument("--no-batch", action="store_true", help="skip the Gemma batched decode (configs[4])")
    ap.add_argument("--no-configs", action="store_true", help="skip configs[0], the M=16/128 sweep and configs[3]")
    ap.add_argument("--batch-steps", type=int, default=32)
    ap.add_argument("--batch-prompt", type=int, default=1024)
    ap.add_argument("--batch-sequences", type=int, default=64,
                    help="--case gemma: sequences in all (8 on one GPU is one rank's share at N = 8)")
    ap.add_argument("--case", default=None, help="profile one product (format:rows:K) or 'decode'")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--profile-region", action="store_true",
                    help="--case llama / gemma: bracket one prefill / one batched step with "
                         "cudaProfilerStart/Stop (for ncu --profile-from-start off)")
    args = ap.parse_args()
    if args.case in ("sweep", "sweep-tensor"):
        print(json.dumps(sweep_bench(flags=2 if args.case == "sweep-tensor" else 0)))
    elif args.case == "sweep-forms":
        ms = [16, 128, 256, 512, 2048]
        for f in (4, 8):
            print(json.dumps(sweep_bench(flags=f, ms=ms, formats=(2,), head=False)))
    elif args.case == "gemma":
        rank, world, local = dist_setup(args.gpus)
        r = gemma_batch_bench(args.batch_steps, world, rank, sequences=args.batch_sequences,
                              prompt_len=args.batch_prompt, cpu=not args.profile_region,
                              profile=args.profile_region)
        if rank == 0:
            print(json.dumps(r))
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    elif args.case == "gemma-split":
        rank, world, local = dist_setup(args.gpus)
        r = gemma_split_bench(args.batch_steps, world, rank, prompt_len=args.batch_prompt)
        if rank == 0:
            print(json.dumps(r))
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    elif args.case == "split-forms":
        print(json.dumps(split_forms_bench()))
    elif args.case == "config1":
        print(json.dumps(config1_bench()))
    elif args.case == "llama":
        import torch
        torch.cuda.set_device(0)
        if args.profile_region:   # the tensor form's prefill alone, for a launch list
            print(json.dumps(llama_bench(4, SEED + 11, cpu=False, forms=(True,), profile=True)))
        else:
            print(json.dumps(llama_bench(128, SEED + 11)))
    elif args.case == "decode":
        import torch
        torch.cuda.set_device(0)
        print(json.dumps(decode_bench(args.decode_steps, 512, SEED + 7, 1)))
    elif args.case:
        run_case(args.case, args.steps)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
