#!/usr/bin/env python3
"""Benchmark: int8-KV decode-attention + append tokens/s on B200.

Workload (the headline): Llama-3.1-8B-shaped
continuous batch — 32 layers, 32 query heads, 8 KV heads, head_dim 128, int8
K/V in groups of 64, 32 concurrent sequences per GPU with ragged lengths
U[512, 8192] (seed 1). One step = append one bf16 token of K/V per
(sequence, layer) + decode attention of one bf16 query per (sequence, layer)
over the whole int8 cache. Data is seeded synthetic N(0,1) (no dataset).

  value  tokens/s over all GPUs, device time (CUDA events), inputs resident
  e2e    the same through the public C ABI with host buffers: pinned
         host->device copy of q/k/v, the call, device->host copy of the
         output, host wall clock
  roofline  the attention kernel's algorithmic bytes / its event time vs the
         measured HBM copy bandwidth (MEASURED_PEAKS.json)
  cpu_baseline  the reference dataflow (quantize, concat copy, full fp16
         dequant, SDPA) restated in C++ (oracle/), timed on this host on a
         bounded sample

Multi-GPU: one process per GPU (torchrun). The global batch is 32 x N
sequences partitioned by longest-processing-time on bytes; no collective on
the data path (weak scaling); timing is the max over ranks.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    # name: layers, hq, hkv, D, G, dtype, seqs/GPU, length sampler, scale
    "llama31_8b_batch32": dict(layers=32, hq=32, hkv=8, D=128, G=64, dtype="bf16", seqs=32,
                               lens=("uniform", 512, 8192, 1), scale=1 / math.sqrt(128)),
    # configs[0] is quoted on 128 decode steps: its default step count
    "llama32_1b_single": dict(layers=16, hq=32, hkv=8, D=64, G=64, dtype="f16", seqs=1,
                              lens=("fixed", 2048, 2048, 0), scale=1 / 8.0, steps=128),
    "qwen3_30b_longctx": dict(layers=48, hq=32, hkv=4, D=128, G=64, dtype="bf16", seqs=16,
                              lens=("fixed", 32768, 32768, 3), scale=1 / math.sqrt(128),
                              values="N(0,0.5)+1%N(0,8)"),
    # 64 requests = one shared 4096-token prefix + a unique 256-token suffix
    # 26 layers = 22 sliding (window 1024) + 4 global, D=256, 256 ragged seqs
    "gemma_mixed_256": dict(layers=26, layers_global=4, layers_sliding=22, window=1024, hq=8, hkv=4,
                            D=256, G=64, dtype="f16", seqs=256, lens=("uniform", 1024, 16384, 5),
                            scale=1.0, shared_prefix=2048, shared_frac=0.3),
    "llama31_8b_prefix64": dict(layers=32, hq=32, hkv=8, D=128, G=64, dtype="bf16", seqs=64,
                                lens=("fixed", 4352, 4352, 2), scale=1 / math.sqrt(128),
                                prefix=4096, suffix=256),
}
# The rows after the decode path (each measured on one GPU, at the
# Llama-3.1-8B KV shape): the prefix-cache disk tier, the fused RoPE append,
# speculative verify and chunked prefill attention.
NEXT_ROWS = {
    "next_prefix_disk": dict(layers=32, hq=32, hkv=8, D=128, G=64, prefix=4096, steps=5),
    "next_rope_append": dict(layers=32, hq=32, hkv=8, D=128, G=64, seqs=32, chunk=256),
    "next_verify4": dict(layers=32, hq=32, hkv=8, D=128, G=64, seqs=32, n_query=4,
                         lens=("uniform", 512, 8192, 1), scale=1 / math.sqrt(128)),
    "next_prefill512": dict(layers=32, hq=32, hkv=8, D=128, G=64, seqs=8, prefix=4096, chunk=512,
                            scale=1 / math.sqrt(128), steps=5),
}
CONFIGS.update(NEXT_ROWS)
DEFAULT_CONFIG = "llama31_8b_batch32"
L2_FLUSH_BYTES = 256 << 20  # 2 x the B200's 126 MB L2, rounded up
# The timed region (K steps) is repeated this many times; `value` comes from
# the median repetition.
REPEATS = 5
# At N > 1 rank 0 stores a prefix entry of this many tokens and every other
# rank imports it over NVLink (outside the timed region) and checks it.
PEER_PREFIX = 4096



def attn_impl_of(args):
    """The pool's attention implementation for --attn-impl."""
    import krill_b200 as kb
    return {"tc": kb.ATTN_TENSOR_CORE, "tcpair": kb.ATTN_TENSOR_CORE_PAIR,
            "cuda": kb.ATTN_CUDA_CORE}[args.attn_impl]

def algo_bytes_attn(L, hkv, D, G):
    return L * hkv * (2 * D + 8 * D // G)


def step_bytes(lengths_after, cfg, raw=False):
    """Algorithmic bytes of one step split into the attention kernel's share
    and the whole step. int8: K/V codes + fp16 scale and zero per group,
    2D + 8D/G bytes per (token, head); raw bf16 pools: 4D."""
    hkv, hq, D, G, layers = cfg["hkv"], cfg["hq"], cfg["D"], cfg["G"], cfg["layers"]
    per_tok = 4 * D if raw else 2 * D + 8 * D // G
    attn = sum(L * hkv * per_tok for L in lengths_after) * layers
    qo = len(lengths_after) * layers * 2 * hq * D * 2
    append = len(lengths_after) * layers * (hkv * D * 4 + hkv * per_tok)
    return attn + qo, attn + qo + append


def kv_randn(torch, cfg, shape, gen, dev):
    """Seeded synthetic K/V in fp32: N(0,1), or for configs[3] N(0, 0.5) with
    1% outliers N(0, 8) (a Bernoulli mask)."""
    x = torch.randn(shape, generator=gen, device=dev, dtype=torch.float32)
    if cfg.get("values") != "N(0,0.5)+1%N(0,8)":
        return x
    x.mul_(math.sqrt(0.5))
    mask = torch.rand(shape, generator=gen, device=dev) < 0.01
    out = torch.randn(shape, generator=gen, device=dev, dtype=torch.float32).mul_(math.sqrt(8.0))
    return torch.where(mask, out, x)


def sample_lengths(cfg, n, seed_offset=0):
    kind, lo, hi, seed = cfg["lens"]
    if kind == "fixed":
        return [lo] * n
    rng = np.random.default_rng(seed + seed_offset)
    return [int(x) for x in rng.integers(lo, hi + 1, size=n)]


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    def __init__(self, device_index):
        self.dev = device_index
        self.rows = []
        self.proc = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", str(self.dev)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            # the timed region starts once sampling is live (nvidia-smi takes
            # a moment to print its first row)
            t0 = time.perf_counter()
            while not self.rows and time.perf_counter() - t0 < 3.0 and self.proc.poll() is None:
                time.sleep(0.01)
            self.first = len(self.rows)
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def __exit__(self, *a):
        if self.proc:
            self.stop = len(self.rows)  # rows printed while the region ran
            time.sleep(0.06)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        # the rows printed while the timed region ran, plus the one that was
        # live when it started
        lo = max(0, getattr(self, "first", 1) - 1)
        rows = self.rows[lo:getattr(self, "stop", len(self.rows)) + 1] or self.rows
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in rows:
            for name, val in zip(names, r[5:9]):
                if val.strip().lower() in ("active", "1"):
                    reasons.add(name)
        pw = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "sm_mhz_min": min(sm) if sm else None,
                "power_w_median": float(np.median(pw)) if pw else None,
                "power_w_max": max(pw) if pw else None,
                "reasons": sorted(reasons), "samples": len(rows)}


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def measured_tensor_peak():
    """Dense bf16 burst TFLOP/s from MEASURED_PEAKS.json (kernels timed alone)."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, "fallback"


def profiled_traffic(workload, algo_bytes):
    """DRAM traffic of one attention launch, from the committed ncu summary of
    this workload (dram bytes read + written per algorithmic byte on a
    smaller capture of the same kernel, scaled to the full launch)."""
    path = os.path.join(ROOT, "profiles", f"attn_tc_kernel_{workload}.md")
    try:
        for line in open(path):
            if line.startswith("traffic_per_algorithmic_byte:"):
                return float(line.split(":")[1]) * algo_bytes
    except OSError:
        pass
    return None


def pinned_copy(torch, t):
    """A page-locked host copy of device tensor `t`."""
    return torch.empty(t.shape, dtype=t.dtype, pin_memory=True).copy_(t.cpu())


def host_step_seconds(torch, dist, world, dev, stream, step_fn, steps):
    """Seconds per step of `step_fn` (public calls whose inputs and outputs
    are host buffers), by the wall clock from the call until the host holds
    the outputs; one untimed step first, mean over `steps`, max over ranks."""
    step_fn()
    stream.synchronize()
    if world > 1:
        dist.barrier()
    total = 0.0
    for _ in range(steps):
        t0 = time.perf_counter()
        step_fn()
        stream.synchronize()
        total += time.perf_counter() - t0
    sec = total / steps
    if world > 1:
        t = torch.tensor([sec], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        sec = float(t.item())
    return sec


def cpu_baseline(cfg, lengths, steps, threads, layer_sample):
    """Time the oracle's reference-dataflow restatement on a bounded sample:
    all sequences, `layer_sample` of the layers, `steps` steps; scaled to the
    full step by layers / layer_sample."""
    import oracle
    n = len(lengths) * layer_sample
    lens = [L for L in lengths for _ in range(layer_sample)]
    base = oracle.Baseline(n, cfg["hkv"], cfg["D"], cfg["G"], lens, steps + 1, seed=7)
    rng = np.random.default_rng(11)
    dt = 1 if cfg["dtype"] == "bf16" else 0
    from tests._data import to_bits
    knew = to_bits(rng.standard_normal((n, cfg["hkv"], cfg["D"]), dtype=np.float32), dt)
    vnew = to_bits(rng.standard_normal((n, cfg["hkv"], cfg["D"]), dtype=np.float32), dt)
    q = to_bits(rng.standard_normal((n, cfg["hq"], cfg["D"]), dtype=np.float32), dt)
    out = np.empty((n, cfg["hq"], cfg["D"]), np.uint16)
    t0 = time.perf_counter()
    for _ in range(steps):
        base.step(knew, vnew, q, cfg["hq"], dt, cfg["scale"], out, threads)
    el = time.perf_counter() - t0
    base.close()
    per_step_full = el / steps * (cfg["layers"] / layer_sample)
    return len(lengths) / per_step_full, el


def headline_config(args, cfg, world, lengths_all, mine, raw):
    """The `config` object of the decode-step workloads' JSON line; the
    reference arm prints the same one."""
    step_b = step_bytes([L + 1 for L in mine], cfg, raw)[1]
    return {"workload": args.config, "kv_format": args.kv, "layers": cfg["layers"], "q_heads": cfg["hq"],
            "kv_heads": cfg["hkv"], "head_dim": cfg["D"], "group_size": cfg["G"],
            "kv_in_dtype": cfg["dtype"], "kv_values": cfg.get("values", "N(0,1)"),
            "seqs_per_gpu": cfg["seqs"], "global_seqs": len(lengths_all),
            "mean_len": float(np.mean(lengths_all)),
            "l2": (f"inputs larger than L2 ({step_b / 1e9:.2f} GB/step)" if step_b >= L2_FLUSH_BYTES
                   else f"L2 flushed between steps ({step_b / 1e9:.3f} GB/step < "
                        f"{L2_FLUSH_BYTES / 1e9:.2f} GB; each step timed alone)"),
            "attn_impl": args.attn_impl, "parallelism": f"seq-partition x{world}"}


def run_reference_arm(args, cfg, rank, world):
    """--impl reference: the reference's CPU dataflow (oracle port), all host
    threads, rank 0 only. The sample is the batch share of one GPU's rank
    (rank 0's sequences): at N GPUs the driver's ratio then compares N GPUs
    with one host's cores on the same per-GPU work."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    from krill_b200.shard import lpt_partition
    lengths_all = sample_lengths(cfg, cfg["seqs"] * world)
    mine = [lengths_all[i] for i in lpt_partition(lengths_all, world)[0]]
    # bounded sample per step: rank 0's sequences, 1 of the layers
    values = []
    t_all = time.perf_counter()
    for _ in range(args.warmup):
        cpu_baseline(cfg, mine, 1, threads, 1)
    for _ in range(args.steps):
        v, _ = cpu_baseline(cfg, mine, 1, threads, 1)
        values.append(v)
    value = float(np.median(values))
    if "prefix" in cfg or "window" in cfg:
        config = {"workload": args.config, "seqs": len(mine), "layers": cfg["layers"]}
    else:
        config = headline_config(args, cfg, world, lengths_all, mine, False)
    line = {
        "impl": "reference", "metric": "int8-KV decode-attn+append tokens/s", "value": value,
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "u8", "data": "synthetic",
        "config": config,
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"{len(mine)} seqs (rank 0's share of {len(lengths_all)}) x 1 of "
                                   f"{cfg['layers']} layers per step, scaled x{cfg['layers']}; oracle/ "
                                   "C++ restatement of QuantizedKVCache.update + SDPA (MLX CPU path "
                                   "unavailable)"},
        "normalisation": ("one host's cores on one GPU rank's share of the batch; at N GPUs the GPU "
                          "arm's value covers all N shares"),
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": time.perf_counter() - t_all,
    }
    print(json.dumps(line), flush=True)


def peer_prefix_check(kb, torch, dist, pool, cfg, rank, world, dev, gen, tdt, stream):
    """N > 1, outside the timed region: rank 0 stores a PEER_PREFIX-token
    prefix entry; every other rank imports it from rank 0's pool over NVLink
    (CUDA IPC handle + entry descriptor, then a peer copy into its own pool,
    krill_prefix_import) and checks that every layer's codes, scales and zeros
    are bit-identical to the owner's (krill_seq_snapshot_quantized on both
    sides; the owner's tensors reach the other ranks by NCCL broadcast).
    Returns this rank's record (None on rank 0)."""
    P, layers, hkv, D = PEER_PREFIX, cfg["layers"], cfg["hkv"], cfg["D"]
    tokens = list(range(1_000_000, 1_000_000 + P))
    pc = kb.PrefixCache(pool)
    obj = [None]
    if rank == 0:
        base = pool.create_sequence()
        for l0 in range(0, layers, 4):
            lc = min(4, layers - l0)
            kb.append_quantize(pool, [base], l0, kv_randn(torch, cfg, (lc, 1, hkv, P, D), gen, dev).to(tdt),
                               kv_randn(torch, cfg, (lc, 1, hkv, P, D), gen, dev).to(tdt))
        pc.store_quantized(tokens, "bench-peer", base)
        base.release()
        entry = pc.lookup_quantized(tokens, "bench-peer")
        torch.cuda.synchronize()
        obj = [(pool.ipc_handle(), pc.describe(entry))]
    dist.broadcast_object_list(obj, src=0)
    rec = None
    if rank != 0:
        handle, desc = obj[0]
        t0 = time.perf_counter()
        entry = pc.import_entry(handle, desc, stream=stream)  # maps rank 0's pool once
        torch.cuda.synchronize()
        first_ms = (time.perf_counter() - t0) * 1e3
        entry.release()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        entry = pc.import_entry(handle, desc, stream=stream)
        e1.record(stream)
        torch.cuda.synchronize()
        nbytes = (P // 256) * pool.block_bytes
        rec = {"rank": rank, "bytes": nbytes, "first_import_ms_incl_mapping": first_ms,
               "copy_ms": e0.elapsed_time(e1), "GB/s": nbytes / (e0.elapsed_time(e1) / 1e3) / 1e9}
    seq = entry.fork(P)
    same = True
    for layer in range(layers):
        snap = seq.quantized_snapshot(layer)
        for t in (snap.keys, snap.values, snap.key_scales, snap.key_zeros, snap.value_scales,
                  snap.value_zeros):
            ref = t.clone() if rank == 0 else torch.empty_like(t)
            dist.broadcast(ref, src=0)
            same = same and torch.equal(ref, t)
    torch.cuda.synchronize()
    seq.release()
    dist.barrier()  # the owner keeps its blocks until every copy is done
    entry.release()
    pc.close()
    if rec is not None:
        rec["bit_identical"] = bool(same)
    return rec


def run_prefix_workload(args, cfg, kb, torch, dist, rank, world, local_rank):
    """shared-prefix reuse. Every rank builds one 4096-token prefix
    (bf16 N(0,1) K/V quantized by the append kernel) and stores it in its
    prefix cache; its requests then look the prefix up (exact-key scan), fork
    its blocks (reference-counted, nothing copied, no prefill of the prefix),
    prefill only their unique 256-token suffix, and run decode steps (append 1
    token + attention per request). Reports decode tokens/s, the logical bytes
    (every request reads its whole cache) and the unique bytes (shared prefix
    blocks counted once per layer per step)."""
    layers, hq, hkv, D, G = cfg["layers"], cfg["hq"], cfg["hkv"], cfg["D"], cfg["G"]
    P, S, n = cfg["prefix"], cfg["suffix"], cfg["seqs"]
    tdt = torch.bfloat16
    dev = torch.device("cuda", local_rank)
    e2e_steps = max(3, args.steps // 2)
    steps_total = args.warmup + REPEATS * args.steps + e2e_steps + 3
    blocks = P // 256 + n * ((P + S + steps_total + 255) // 256 - P // 256 + 1) + 4
    pool = kb.KVPool(layers, hkv, hq, D, num_blocks=blocks, group_size=G, device=local_rank,
                     attn_impl=attn_impl_of(args))
    pc = kb.PrefixCache(pool)
    gen = torch.Generator(device=dev)
    gen.manual_seed(4321 + rank)
    base = pool.create_sequence()
    k = torch.randn((layers, 1, hkv, P, D), generator=gen, device=dev).to(tdt)
    v = torch.randn((layers, 1, hkv, P, D), generator=gen, device=dev).to(tdt)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    kb.append_quantize(pool, [base], 0, k, v)
    torch.cuda.synchronize()
    prefix_prefill_s = time.perf_counter() - t0
    prefix_tokens = list(range(P))
    pc.store_quantized(prefix_tokens, "llama-3.1-8b", base)
    # lookup + fork per request (host), then the suffix prefill (device)
    t0 = time.perf_counter()
    seqs, hits = [], 0
    for r in range(n):
        prompt = prefix_tokens + [1_000_000 + r * S + i for i in range(S)]
        hit = pc.lookup_quantized(prompt, "llama-3.1-8b")
        if hit is None:
            hit = pc.lookup_longest_prefix_quantized(prompt, "llama-3.1-8b")
        hits += hit is not None and hit.prefix_length == P
        seqs.append(hit.fork(min(hit.prefix_length, len(prompt) - 1)))
        hit.release()
    lookup_fork_us = (time.perf_counter() - t0) / n * 1e6
    refcount = pool.refcount(base.blocks()[0])
    ks = torch.randn((layers, n, hkv, S, D), generator=gen, device=dev).to(tdt)
    vs = torch.randn((layers, n, hkv, S, D), generator=gen, device=dev).to(tdt)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    kb.append_quantize(pool, seqs, 0, ks, vs)
    torch.cuda.synchronize()
    suffix_prefill_s = time.perf_counter() - t0
    del k, v, ks, vs
    k1 = torch.randn((layers, n, hkv, 1, D), generator=gen, device=dev).to(tdt)
    v1 = torch.randn((layers, n, hkv, 1, D), generator=gen, device=dev).to(tdt)
    q = torch.randn((layers, n, hq, D), generator=gen, device=dev).to(tdt)
    out = torch.empty((layers, n, hq, D), dtype=tdt, device=dev)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        kb.decode_step(pool, seqs, 0, k1, v1, q, out, cfg["scale"], stream=stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    len0 = seqs[0].length(0)
    pool.set_profiling(True)
    pool.kernel_times()
    pool.kernel_count()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = []
    with ClockSampler(local_rank) as clocks:
        for _ in range(REPEATS):
            torch.cuda.synchronize()
            start.record(stream)
            for _ in range(args.steps):
                kb.decode_step(pool, seqs, 0, k1, v1, q, out, cfg["scale"], stream=stream)
            stop.record(stream)
            torch.cuda.synchronize()
            ms = start.elapsed_time(stop) / args.steps
            if world > 1:
                t = torch.tensor([ms], dtype=torch.float64, device=dev)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                ms = float(t.item())
            reps.append(ms)
    if world > 1:
        dist.barrier()
    am, an, pm, pn = pool.kernel_times()
    launches = pool.kernel_count() // REPEATS
    pool.set_profiling(False)
    # end to end: the same step through krill_decode_step_host with
    # page-locked host inputs and output
    h_k, h_v, h_q = pinned_copy(torch, k1), pinned_copy(torch, v1), pinned_copy(torch, q)
    h_out = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    e2e_s = host_step_seconds(
        torch, dist, world, dev, stream,
        lambda: kb.decode_step_host(pool, seqs, 0, h_k, h_v, h_q, h_out, cfg["scale"], stream=stream),
        e2e_steps)
    h2d = sum(t.numel() * t.element_size() for t in (h_k, h_v, h_q))
    d2h = h_out.numel() * h_out.element_size()
    ms = float(np.median(reps))
    per_tok = hkv * (2 * D + 8 * D // G)
    mean_len = len0 + (REPEATS * args.steps + 1) / 2
    logical = n * layers * mean_len * per_tok + n * layers * 2 * hq * D * 2
    unique = layers * (P + n * (mean_len - P)) * per_tok + n * layers * 2 * hq * D * 2
    attn_ms = am / max(1, an)
    peak, peak_kind = measured_peak()
    if rank == 0:
        line = {
            "metric": "int8-KV decode-attn+append tokens/s (shared-prefix batch)",
            "value": n * world / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8",
            "data": "synthetic",
            "config": {"workload": args.config, "requests_per_gpu": n, "prefix": P, "suffix": S,
                       "layers": layers, "kv_heads": hkv, "head_dim": D, "group_size": G},
            "prefix": {"hits": hits, "requests": n, "lookup_fork_us_per_request": lookup_fork_us,
                       "prefix_block_refcount": refcount, "prefix_prefill_s": prefix_prefill_s,
                       "suffix_prefill_s": suffix_prefill_s,
                       "prefill_tokens_skipped_per_request": P,
                       "gather_bytes_copied": 0,
                       "reference_style_copy_bytes_per_request": layers * P * per_tok},
            "roofline": {"bound": "hbm", "kernel": "attn_tc_kernel", "attn_ms": attn_ms,
                         "append_ms": pm / max(1, pn),
                         "achieved_logical": logical / (attn_ms / 1e3) / 1e9,
                         "achieved_unique": unique / (attn_ms / 1e3) / 1e9,
                         "peak": peak, "unit": "GB/s", "peak_kind": peak_kind,
                         "frac_unique": unique / (attn_ms / 1e3) / 1e9 / peak,
                         "algo_bytes_logical": logical, "algo_bytes_unique": unique},
            "e2e": {"value": n * world / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "api": "krill_decode_step_host",
                    "ms_per_step": e2e_s * 1e3, "steps": e2e_steps},
            "gpu_launches": launches,
            "clocks": clocks.summary(),
            "ms_per_step_repeats": reps,
            "device_error_flag": pool.device_error(),
        }
        print(json.dumps(line), flush=True)
    pc.close()
    pool.close()
    if world > 1:
        dist.destroy_process_group()


def run_next_row(args, cfg, kb, torch, rank, world, local_rank):
    """The rows after the decode path, one GPU each (rank 0; other ranks exit):
    - next_prefix_disk: a 4096-token entry stored to the disk tier (gather +
      safetensors write, write-behind then waited for) and served after a
      restart (a fresh cache on the same directory: file read + restore
      kernel into pool blocks); GB/s of entry bytes each way.
    - next_rope_append: 256-token chunks appended to 32 sequences with the
      fused RoPE (krill_append_quantize_rope) and without it; appended
      tokens/s and HBM GB/s of the append kernel.
    - next_verify4: speculative verify of 4 tokens per sequence (append 4, then
      krill_verify_attention with n_query = 4) over the configs[1] batch;
      verified tokens/s against the unique cache bytes.
    - next_prefill512: 512-token chunks of prefill over a 4096-token int8
      cache per sequence (append the chunk, then krill_prefill_attention);
      prefill tokens/s and tensor FLOP/s of the causal attention."""
    if rank != 0:
        return
    import tempfile, shutil
    layers, hq, hkv, D, G = cfg["layers"], cfg["hq"], cfg["hkv"], cfg["D"], cfg["G"]
    per_tok = hkv * (2 * D + 8 * D // G)  # int8 codes + f16 scales/zeros per token-layer
    dev = torch.device("cuda", local_rank)
    gen = torch.Generator(device=dev)
    gen.manual_seed(99)
    stream = torch.cuda.current_stream()
    peak, peak_kind = measured_peak()
    base = {"n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "data": "synthetic"}

    def rnd(*shape):
        return torch.randn(shape, generator=gen, device=dev).to(torch.bfloat16)

    if args.config == "next_prefix_disk":
        P = cfg["prefix"]
        pool = kb.KVPool(layers, hkv, hq, D, num_blocks=3 * P // 256 + 8, group_size=G, device=local_rank)
        d = tempfile.mkdtemp(prefix="krill_disk_")
        try:
            src = pool.create_sequence()
            kb.append_quantize(pool, [src], 0, rnd(layers, 1, hkv, P, D), rnd(layers, 1, hkv, P, D))
            torch.cuda.synchronize()
            entry_bytes = layers * P * per_tok
            w_s, r_s = [], []
            for i in range(args.warmup + args.steps):
                toks = [i * 1_000_000 + t for t in range(P)]
                pc = kb.PrefixCache(pool, cache_dir=d, disk_budget_bytes=-1)
                t0 = time.perf_counter()
                pc.store_quantized(toks, "m", src)
                pc.wait_for_disk_writes()
                t1 = time.perf_counter()
                pc.close()
                pc2 = kb.PrefixCache(pool, cache_dir=d, disk_budget_bytes=-1)  # after a restart
                t2 = time.perf_counter()
                hit = pc2.lookup_quantized(toks, "m")
                torch.cuda.synchronize()
                t3 = time.perf_counter()
                assert hit is not None and hit.prefix_length == P, "disk tier missed"
                hit.release()
                pc2.close()
                if i >= args.warmup:
                    w_s.append(t1 - t0)
                    r_s.append(t3 - t2)
            w, r = float(np.mean(w_s)), float(np.mean(r_s))
            line = dict(metric="prefix-cache disk tier restore GB/s (restart hit)",
                        value=entry_bytes / r / 1e9, unit="GB/s", ms_per_step=r * 1e3,
                        dtype="u8", **base,
                        config={"workload": args.config, "prefix_tokens": P, "layers": layers,
                                "kv_heads": hkv, "head_dim": D, "group_size": G,
                                "entry_bytes": entry_bytes, "file_system": "tempfile.mkdtemp() on the box"},
                        write={"GBps": entry_bytes / w / 1e9, "ms": w * 1e3},
                        roofline=None,
                        note="host-bound (file I/O and page cache); the restore kernel's HBM work is a small part")
            print(json.dumps(line), flush=True)
        finally:
            shutil.rmtree(d, ignore_errors=True)
            pool.close()
        return

    if args.config == "next_rope_append":
        n, C = cfg["seqs"], cfg["chunk"]
        total = (args.warmup + args.steps) * C
        rows = total + C
        pos = torch.arange(rows, device=dev, dtype=torch.float64)
        inv = 10000.0 ** (-torch.arange(0, D, 2, device=dev, dtype=torch.float64) / D)
        ang = pos[:, None] * inv[None, :]
        cos, sin = torch.cos(ang).float().contiguous(), torch.sin(ang).float().contiguous()
        k, v = rnd(layers, n, hkv, C, D), rnd(layers, n, hkv, C, D)
        res = {}
        for mode in ("rope", "plain"):
            pool = kb.KVPool(layers, hkv, hq, D, num_blocks=n * ((total + 255) // 256 + 1) + 4,
                             group_size=G, device=local_rank)
            seqs = [pool.create_sequence() for _ in range(n)]
            rope = (cos, sin) if mode == "rope" else None
            for _ in range(args.warmup):
                kb.append_quantize(pool, seqs, 0, k, v, stream=stream, rope=rope)
            torch.cuda.synchronize()
            pool.set_profiling(True)
            pool.kernel_times()
            pool.kernel_count()
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with ClockSampler(local_rank) as clocks:
                ev0.record(stream)
                for _ in range(args.steps):
                    kb.append_quantize(pool, seqs, 0, k, v, stream=stream, rope=rope)
                ev1.record(stream)
                torch.cuda.synchronize()
            _, _, app_total, app_n = pool.kernel_times()
            res[mode] = dict(ms=ev0.elapsed_time(ev1) / args.steps, kernel_ms=app_total / max(1, app_n),
                             launches=pool.kernel_count(), clocks=clocks.summary(),
                             err=pool.device_error())
            pool.close()
        tokens = n * C
        algo = tokens * layers * (hkv * D * 2 * 2 + per_tok)  # read new K, V bf16; write codes + meta
        r = res["rope"]
        line = dict(metric="fused RoPE + int8 quantize + append tokens/s", value=tokens / (r["ms"] / 1e3),
                    unit="tokens/s", ms_per_step=r["ms"], dtype="u8", **base,
                    config={"workload": args.config, "seqs": n, "chunk_tokens": C, "layers": layers,
                            "kv_heads": hkv, "head_dim": D, "group_size": G, "kv_in_dtype": "bf16",
                            "rope": "rotate-half, base 10000, caller-owned f32 cos/sin table"},
                    roofline={"bound": "hbm", "kernel": "append_rows_kernel (RoPE)",
                              "achieved": algo / (r["kernel_ms"] / 1e3) / 1e9, "peak": peak,
                              "unit": "GB/s", "peak_kind": peak_kind,
                              "frac": algo / (r["kernel_ms"] / 1e3) / 1e9 / peak,
                              "algo_bytes": algo, "kernel_ms": r["kernel_ms"]},
                    plain_append={"tokens_per_s": tokens / (res["plain"]["ms"] / 1e3),
                                  "kernel_ms": res["plain"]["kernel_ms"],
                                  "frac": algo / (res["plain"]["kernel_ms"] / 1e3) / 1e9 / peak},
                    gpu_launches=r["launches"], clocks=r["clocks"], device_error_flag=r["err"])
        print(json.dumps(line), flush=True)
        return

    if args.config == "next_verify4":
        n, nq = cfg["seqs"], cfg["n_query"]
        lens = sample_lengths(cfg, n)
        total_new = (args.warmup + args.steps) * nq
        pool = kb.KVPool(layers, hkv, hq, D, num_blocks=sum((L + total_new + 255) // 256 for L in lens) + 4,
                         group_size=G, device=local_rank)
        seqs = [pool.create_sequence() for _ in lens]
        for s_, L in zip(seqs, lens):
            for l0 in range(0, layers, 8):
                kb.append_quantize(pool, [s_], l0, rnd(8, 1, hkv, L, D), rnd(8, 1, hkv, L, D))
        k1, v1 = rnd(layers, n, hkv, nq, D), rnd(layers, n, hkv, nq, D)
        q = rnd(layers, n, nq, hq, D)
        out = torch.empty_like(q)
        for _ in range(args.warmup):
            kb.append_quantize(pool, seqs, 0, k1, v1, stream=stream)
            kb.verify_attention(pool, seqs, 0, q, out, cfg["scale"], stream=stream)
        torch.cuda.synchronize()
        len0 = [s_.length(0) for s_ in seqs]
        pool.set_profiling(True)
        pool.kernel_times()
        pool.kernel_count()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local_rank) as clocks:
            ev0.record(stream)
            for _ in range(args.steps):
                kb.append_quantize(pool, seqs, 0, k1, v1, stream=stream)
                kb.verify_attention(pool, seqs, 0, q, out, cfg["scale"], stream=stream)
            ev1.record(stream)
            torch.cuda.synchronize()
        am, an, _, _ = pool.kernel_times()
        ms = ev0.elapsed_time(ev1) / args.steps
        attn_ms = am / max(1, an)
        # unique bytes: each sequence's cache once per layer (lengths after the
        # step's append), plus q and out; logical: query j reads its prefix
        uniq, logical = 0.0, 0.0
        for i in range(args.steps):
            for L0 in len0:
                L = L0 + (i + 1) * nq
                uniq += layers * (L * per_tok + 2 * nq * hq * D * 2)
                logical += layers * (sum(L - nq + 1 + j for j in range(nq)) * per_tok + 2 * nq * hq * D * 2)
        uniq /= args.steps
        logical /= args.steps
        line = dict(metric="int8-KV speculative verify tokens/s (4 queries per sequence)",
                    value=n * nq / (ms / 1e3), unit="tokens/s", ms_per_step=ms, dtype="u8", **base,
                    config={"workload": args.config, "seqs": n, "n_query": nq, "layers": layers,
                            "q_heads": hq, "kv_heads": hkv, "head_dim": D, "group_size": G,
                            "mean_len": float(np.mean(lens)), "path": "decode kernel, query tiles of 8 columns (up to 2 per unit), each column one (query, head) (n_query x GQA < 64 rows)"},
                    roofline={"bound": "hbm", "kernel": "attn_tc_kernel", "attn_ms": attn_ms,
                              "achieved_unique": uniq / (attn_ms / 1e3) / 1e9,
                              "achieved_logical": logical / (attn_ms / 1e3) / 1e9,
                              "peak": peak, "unit": "GB/s", "peak_kind": peak_kind,
                              "frac_unique": uniq / (attn_ms / 1e3) / 1e9 / peak,
                              "frac_logical": logical / (attn_ms / 1e3) / 1e9 / peak,
                              "algo_bytes_unique": uniq, "algo_bytes_logical": logical},
                    gpu_launches=pool.kernel_count(), clocks=clocks.summary(),
                    device_error_flag=pool.device_error())
        pool.close()
        print(json.dumps(line), flush=True)
        return

    if args.config == "next_prefill512":
        n, P, C = cfg["seqs"], cfg["prefix"], cfg["chunk"]
        # each step takes two of the library's 16 metadata staging slots, and
        # a slot grows (a pinned host allocation) the first time it holds a
        # step's large packet: warm up until every slot has been used
        warmup = max(args.warmup, 9)
        total = P + (warmup + args.steps) * C
        pool = kb.KVPool(layers, hkv, hq, D, num_blocks=n * ((total + 255) // 256 + 1) + 4, group_size=G,
                         device=local_rank, attn_impl=attn_impl_of(args))
        seqs = [pool.create_sequence() for _ in range(n)]
        for s_ in seqs:
            for l0 in range(0, layers, 8):
                kb.append_quantize(pool, [s_], l0, rnd(8, 1, hkv, P, D), rnd(8, 1, hkv, P, D))
        kc, vc = rnd(layers, n, hkv, C, D), rnd(layers, n, hkv, C, D)
        q = rnd(layers, n, C, hq, D)
        out = torch.empty_like(q)
        for _ in range(warmup):
            kb.append_quantize(pool, seqs, 0, kc, vc, stream=stream)
            kb.prefill_attention(pool, seqs, 0, q, out, cfg["scale"], stream=stream)
        torch.cuda.synchronize()
        len0 = seqs[0].length(0)
        pool.set_profiling(True)
        pool.kernel_times()
        pool.kernel_count()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local_rank) as clocks:
            ev0.record(stream)
            for _ in range(args.steps):
                kb.append_quantize(pool, seqs, 0, kc, vc, stream=stream)
                kb.prefill_attention(pool, seqs, 0, q, out, cfg["scale"], stream=stream)
            ev1.record(stream)
            torch.cuda.synchronize()
        am, an, pm, pn = pool.kernel_times()
        ms = ev0.elapsed_time(ev1) / args.steps
        attn_ms = am / max(1, an)
        # causal attention FLOPs: query j of a chunk ending at length L sees
        # L - C + j + 1 keys; q·kᵀ and p·v are 2·D FLOPs each per (query head, key)
        flops = 0.0
        for i in range(args.steps):
            L = len0 + (i + 1) * C
            keys = C * (L - C) + C * (C + 1) / 2
            flops += n * layers * hq * 4 * D * keys
        flops /= args.steps
        tpeak, tpeak_kind = measured_tensor_peak()
        line = dict(metric="int8-KV chunked-prefill attention tokens/s (512-token chunks)",
                    value=n * C / (ms / 1e3), unit="tokens/s", ms_per_step=ms, dtype="u8", **base,
                    config={"workload": args.config, "seqs": n, "prefix_tokens": P, "chunk_tokens": C,
                            "layers": layers, "q_heads": hq, "kv_heads": hkv, "head_dim": D,
                            "group_size": G, "path": "causal tcgen05 cascade items"},
                    roofline={"bound": "tensor", "kernel": "attn_shared_umma_kernel (causal)",
                              "attn_ms": attn_ms, "append_ms": pm / max(1, pn),
                              "achieved": flops / (attn_ms / 1e3) / 1e12, "peak": tpeak,
                              "unit": "TFLOP/s", "peak_kind": tpeak_kind,
                              "frac": flops / (attn_ms / 1e3) / 1e12 / tpeak, "algo_flops": flops},
                    gpu_launches=pool.kernel_count(), clocks=clocks.summary(),
                    device_error_flag=pool.device_error())
        line["warmup"] = warmup
        pool.close()
        print(json.dumps(line), flush=True)
        return


def run_mixed_workload(args, cfg, kb, torch, dist, rank, world, local_rank):
    """mixed local/global cache. Two pools per GPU: the 4 global
    layers (full history) and the 22 sliding layers (window 1024, ring of
    blocks, RotatingKVCache semantics). 256 sequences per GPU with lengths
    U[1024, 16384]; 30% of them fork a shared 2048-token prefix in the global
    pool (in the sliding layers the prefix's window is overwritten once a
    sequence is 1024 tokens past it). One step = append + attention in both
    pools. The cache is filled with f16 N(0,1) K/V through the append kernel;
    the sliding layers receive every token of each sequence, 256 per call, so
    their rings have wrapped as in a long-running request."""
    from krill_b200.shard import lpt_partition
    Lg, Ls, W = cfg["layers_global"], cfg["layers_sliding"], cfg["window"]
    hq, hkv, D, G = cfg["hq"], cfg["hkv"], cfg["D"], cfg["G"]
    n_total = cfg["seqs"] * world
    lengths_all = sample_lengths(cfg, n_total)
    mine = [lengths_all[i] for i in lpt_partition(lengths_all, world)[rank]]
    n = len(mine)
    rng = np.random.default_rng(17)
    shared = set(i for i in range(n) if rng.random() < cfg["shared_frac"] and mine[i] > cfg["shared_prefix"])
    P = cfg["shared_prefix"]
    dev = torch.device("cuda", local_rank)
    e2e_steps = max(3, args.steps // 2)
    steps_total = args.warmup + REPEATS * args.steps + e2e_steps + 3
    blocks_g = sum((L + steps_total + 255) // 256 for L in mine) + 8
    glob = kb.KVPool(Lg, hkv, hq, D, num_blocks=blocks_g, group_size=G, device=local_rank)
    slid = kb.KVPool(Ls, hkv, hq, D, num_blocks=n * 5 + 8, group_size=G, window=W, max_append=256,
                     device=local_rank)
    pc = kb.PrefixCache(glob)
    gen = torch.Generator(device=dev)
    gen.manual_seed(999 + rank)
    maxL = max(mine)
    bufk = torch.randn((Lg * hkv * maxL * D,), generator=gen, device=dev).to(torch.float16)
    bufv = torch.randn((Lg * hkv * maxL * D,), generator=gen, device=dev).to(torch.float16)

    def chunk(buf, lc, L):
        return buf[: lc * hkv * L * D].view(lc, 1, hkv, L, D)

    t_fill = time.perf_counter()
    stream = torch.cuda.current_stream()
    # the shared prefix is owned by GPU 0; other GPUs fetch it once over NVLink
    # (IPC handle + entry descriptor, then a peer copy into the local pool)
    if world == 1 or rank == 0:
        base = glob.create_sequence()
        kb.append_quantize(glob, [base], 0, chunk(bufk, Lg, P), chunk(bufv, Lg, P))
        pc.store_quantized(list(range(P)), "gemma", base)
    peer = None
    if world > 1:
        obj = [None]
        if rank == 0:
            hit0 = pc.lookup_quantized(list(range(P)), "gemma")
            torch.cuda.synchronize()
            obj = [(glob.ipc_handle(), pc.describe(hit0))]
        dist.broadcast_object_list(obj, src=0)
        if rank != 0:
            handle, desc = obj[0]
            # the first import maps the owner's pool (cudaIpcOpenMemHandle,
            # host side); the second, timed on the device, is the NVLink copy
            t0 = time.perf_counter()
            imp = pc.import_entry(handle, desc, stream=stream)
            torch.cuda.synchronize()
            first_ms = (time.perf_counter() - t0) * 1e3
            imp.release()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            imp = pc.import_entry(handle, desc, stream=stream)
            e1.record(stream)
            torch.cuda.synchronize()
            nbytes = ((P + 255) // 256) * glob.block_bytes
            peer = {"rank": rank, "bytes": nbytes, "first_import_ms_incl_mapping": first_ms,
                    "copy_ms": e0.elapsed_time(e1), "GB/s": nbytes / (e0.elapsed_time(e1) / 1e3) / 1e9}
            imp.release()  # the cache keeps the entry
        dist.barrier()  # the owner keeps its blocks until every copy is done
        if rank == 0:
            hit0.release()
    gseqs, sseqs = [], []
    for i, L in enumerate(mine):
        if i in shared:
            prompt = list(range(P)) + [7_000_000 + i]
            hit = pc.lookup_quantized(prompt, "gemma") or pc.lookup_longest_prefix_quantized(prompt, "gemma")
            s = hit.fork(P)
            hit.release()
            kb.append_quantize(glob, [s], 0, chunk(bufk, Lg, L - P), chunk(bufv, Lg, L - P))
        else:
            s = glob.create_sequence()
            kb.append_quantize(glob, [s], 0, chunk(bufk, Lg, L), chunk(bufv, Lg, L))
        gseqs.append(s)
    sk = torch.randn((Ls * hkv * 256 * D,), generator=gen, device=dev).to(torch.float16)
    sv = torch.randn((Ls * hkv * 256 * D,), generator=gen, device=dev).to(torch.float16)
    for L in mine:
        s = slid.create_sequence()
        for t0 in range(0, L, 256):  # every token, 256 per call: the ring wraps
            nt = min(256, L - t0)
            kb.append_quantize(slid, [s], 0, chunk(sk, Ls, nt), chunk(sv, Ls, nt))
        sseqs.append(s)
    del bufk, bufv
    torch.cuda.synchronize()
    t_fill = time.perf_counter() - t_fill
    kg = torch.randn((Lg, n, hkv, 1, D), generator=gen, device=dev).to(torch.float16)
    ks = torch.randn((Ls, n, hkv, 1, D), generator=gen, device=dev).to(torch.float16)
    qg = torch.randn((Lg, n, hq, D), generator=gen, device=dev).to(torch.float16)
    qs = torch.randn((Ls, n, hq, D), generator=gen, device=dev).to(torch.float16)
    og, os_ = torch.empty_like(qg), torch.empty_like(qs)

    def step():
        kb.decode_step(glob, gseqs, 0, kg, kg, qg, og, cfg["scale"], stream=stream)
        kb.decode_step(slid, sseqs, 0, ks, ks, qs, os_, cfg["scale"], stream=stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    lg0 = [s.length(0) for s in gseqs]
    glob.set_profiling(True)
    slid.set_profiling(True)
    glob.kernel_times()
    slid.kernel_times()
    glob.kernel_count()
    slid.kernel_count()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = []
    with ClockSampler(local_rank) as clocks:
        for _ in range(REPEATS):
            torch.cuda.synchronize()
            start.record(stream)
            for _ in range(args.steps):
                step()
            stop.record(stream)
            torch.cuda.synchronize()
            ms = start.elapsed_time(stop) / args.steps
            if world > 1:
                t = torch.tensor([ms], dtype=torch.float64, device=dev)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                ms = float(t.item())
            reps.append(ms)
    if world > 1:
        dist.barrier()
    ms = float(np.median(reps))
    launches = (glob.kernel_count() + slid.kernel_count()) // REPEATS
    ag, _, pg, _ = glob.kernel_times()
    as_, _, ps, _ = slid.kernel_times()
    ag, pg, as_, ps = ag / REPEATS, pg / REPEATS, as_ / REPEATS, ps / REPEATS
    glob.set_profiling(False)
    slid.set_profiling(False)
    # end to end: both pools' steps through krill_decode_step_host with
    # page-locked host inputs and outputs
    hkg, hks = pinned_copy(torch, kg), pinned_copy(torch, ks)
    hqg, hqs = pinned_copy(torch, qg), pinned_copy(torch, qs)
    hog = torch.empty(og.shape, dtype=og.dtype, pin_memory=True)
    hos = torch.empty(os_.shape, dtype=os_.dtype, pin_memory=True)

    def host_step():
        kb.decode_step_host(glob, gseqs, 0, hkg, hkg, hqg, hog, cfg["scale"], stream=stream)
        kb.decode_step_host(slid, sseqs, 0, hks, hks, hqs, hos, cfg["scale"], stream=stream)

    e2e_s = host_step_seconds(torch, dist, world, dev, stream, host_step, e2e_steps)
    # K and V of a step are the same host tensor, copied once per use
    h2d = sum(2 * t.numel() * t.element_size() for t in (hkg, hks))
    h2d += sum(t.numel() * t.element_size() for t in (hqg, hqs))
    d2h = sum(t.numel() * t.element_size() for t in (hog, hos))
    per_tok = hkv * (2 * D + 8 * D // G)
    mid = (REPEATS * args.steps + 1) / 2
    glob_b = sum(L + mid for L in lg0) * Lg * per_tok
    glob_unique = glob_b - len(shared) * P * Lg * per_tok + P * Lg * per_tok
    slid_b = n * min(W, W) * Ls * per_tok
    qo = n * (Lg + Ls) * 2 * hq * D * 2
    attn_ms = (ag + as_) / args.steps
    peak, peak_kind = measured_peak()
    fetches = [None] * world
    if world > 1:
        dist.all_gather_object(fetches, peer)
    if rank == 0:
        line = {
            "metric": "int8-KV decode-attn+append tokens/s (mixed sliding/global)",
            "value": n_total / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8",
            "data": "synthetic",
            "config": {"workload": args.config, "seqs_per_gpu": n, "global_layers": Lg,
                       "sliding_layers": Ls, "window": W, "head_dim": D, "kv_heads": hkv,
                       "q_heads": hq, "shared_prefix_seqs": len(shared),
                       "mean_len": float(np.mean(lengths_all))},
            "roofline": {"bound": "hbm", "kernel": "attn_tc_kernel", "attn_ms": attn_ms,
                         "attn_ms_global": ag / args.steps, "attn_ms_sliding": as_ / args.steps,
                         "append_ms": (pg + ps) / args.steps,
                         "achieved": (glob_b + slid_b + qo) / (attn_ms / 1e3) / 1e9,
                         "achieved_unique": (glob_unique + slid_b + qo) / (attn_ms / 1e3) / 1e9,
                         "peak": peak, "unit": "GB/s", "peak_kind": peak_kind,
                         "frac": (glob_b + slid_b + qo) / (attn_ms / 1e3) / 1e9 / peak,
                         "algo_bytes": glob_b + slid_b + qo},
            "e2e": {"value": n_total / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "api": "krill_decode_step_host",
                    "ms_per_step": e2e_s * 1e3, "steps": e2e_steps},
            "gpu_launches": launches, "fill_s": t_fill, "clocks": clocks.summary(),
            "ms_per_step_repeats": reps,
            "plan_sliding": {"plan": list(slid.last_plan()), "kernels": slid.last_kernels()},
            "plan_global": {"plan": list(glob.last_plan()), "kernels": glob.last_kernels()},
            "prefix_peer_fetch": [f for f in fetches if f],
            "device_error_flag": glob.device_error() | slid.device_error(),
        }
        print(json.dumps(line), flush=True)
    pc.close()
    glob.close()
    slid.close()
    if world > 1:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default 20; the workload's own count where it has one)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="krill", choices=["krill", "reference"])
    ap.add_argument("--config", default=DEFAULT_CONFIG, choices=sorted(CONFIGS))
    ap.add_argument("--attn-impl", default="tc", choices=["tc", "tcpair", "cuda"],
                    help="tc: tensor cores (tcgen05 cascade, one CTA per item); tcpair: the "
                         "cascade on CTA pairs where items have > 128 rows; cuda: CUDA-core decode")
    ap.add_argument("--kv", default="int8", choices=["int8", "bf16"],
                    help="pool format; bf16 = the unquantized comparison variant (default workload)")
    ap.add_argument("--split-tokens", type=int, default=0)
    ap.add_argument("--e2e-chunk", type=int, default=0,
                    help="layers per chunk of the host-buffer step (0 = one chunk)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-layer-sample", type=int, default=12)
    ap.add_argument("--seqs", type=int, default=0, help="override sequences per GPU (profiling)")
    ap.add_argument("--layers", type=int, default=0,
                    help="override the layer count (profiling captures on a smaller pool)")
    ap.add_argument("--diag", action="store_true",
                    help="per-rank, per-step kernel times and device error flags on stderr")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = CONFIGS[args.config].get("steps", 20)
    args.warmup = max(3, args.warmup)
    cfg = dict(CONFIGS[args.config])
    if args.seqs:
        cfg["seqs"] = args.seqs
    if args.layers:
        cfg["layers"] = args.layers

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if args.config in NEXT_ROWS:
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "no CPU restatement is timed for "
                                  "the rows after the decode path; their oracles are test-only"}),
                      flush=True)
            return
        run_reference_arm(args, cfg, rank, world)
        return

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local_rank)
    if world > 1:
        from datetime import timedelta
        # stdout carries exactly one JSON line: while NCCL initialises (its
        # version banner is printed to stdout when the environment sets
        # NCCL_DEBUG=VERSION), file descriptor 1 points at stderr
        sys.stdout.flush()
        saved_stdout = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                    device_id=torch.device("cuda", local_rank))
            # first collective up front, so NCCL's lazy setup never overlaps our kernels
            warm = torch.ones(1, device=torch.device("cuda", local_rank))
            dist.all_reduce(warm)
            torch.cuda.synchronize()
        finally:
            sys.stdout.flush()
            os.dup2(saved_stdout, 1)
            os.close(saved_stdout)

    import krill_b200 as kb

    if args.config in NEXT_ROWS:
        run_next_row(args, cfg, kb, torch, rank, world, local_rank)
        if world > 1:
            dist.destroy_process_group()
        return
    if "prefix" in cfg:
        run_prefix_workload(args, cfg, kb, torch, dist, rank, world, local_rank)
        return
    if "window" in cfg:
        run_mixed_workload(args, cfg, kb, torch, dist, rank, world, local_rank)
        return

    # ---- workload: global batch partitioned over ranks ----
    n_total = cfg["seqs"] * world
    lengths_all = sample_lengths(cfg, n_total)
    from krill_b200.shard import lpt_partition
    parts = lpt_partition(lengths_all, world)
    mine = [lengths_all[i] for i in parts[rank]]
    layers, hq, hkv, D, G = cfg["layers"], cfg["hq"], cfg["hkv"], cfg["D"], cfg["G"]
    tdt = torch.bfloat16 if cfg["dtype"] == "bf16" else torch.float16
    total_steps = args.warmup + args.steps + 4  # repetitions rewind to the same lengths
    # at N > 1 the pool also holds the prefix entry: rank 0's original, or on
    # the other ranks the two imports (the first, kept by the prefix cache,
    # and the timed one) until the check ends
    blocks = sum((L + total_steps + 255) // 256 for L in mine) + 4 + (2 * PEER_PREFIX // 256 + 2 if world > 1 else 0)
    raw = args.kv == "bf16"
    if raw and cfg["dtype"] != "bf16":
        raise SystemExit("--kv bf16 needs a workload with bf16 K/V")
    pool = kb.KVPool(layers, hkv, hq, D, num_blocks=blocks, group_size=G,
                     attn_impl=attn_impl_of(args),
                     split_tokens=args.split_tokens, kv_format=kb.KV_BF16 if raw else kb.KV_INT8,
                     device=local_rank)
    seqs = [pool.create_sequence() for _ in mine]
    dev = torch.device("cuda", local_rank)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    t_fill = time.perf_counter()
    chunk_layers = 4
    for s, L in zip(seqs, mine):
        for l0 in range(0, layers, chunk_layers):
            lc = min(chunk_layers, layers - l0)
            k = kv_randn(torch, cfg, (lc, 1, hkv, L, D), gen, dev).to(tdt)
            v = kv_randn(torch, cfg, (lc, 1, hkv, L, D), gen, dev).to(tdt)
            kb.append_quantize(pool, [s], l0, k, v)
            del k, v
    torch.cuda.synchronize()
    t_fill = time.perf_counter() - t_fill
    stream = torch.cuda.current_stream()
    peer = None
    if world > 1:
        peer = peer_prefix_check(kb, torch, dist, pool, cfg, rank, world, dev, gen, tdt, stream)

    n = len(seqs)
    k_new = kv_randn(torch, cfg, (layers, n, hkv, 1, D), gen, dev).to(tdt)
    v_new = kv_randn(torch, cfg, (layers, n, hkv, 1, D), gen, dev).to(tdt)
    q = torch.randn((layers, n, hq, D), generator=gen, device=dev).to(tdt)
    out = torch.empty((layers, n, hq, D), dtype=tdt, device=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-timed region: inputs resident in HBM ----
    if args.diag:
        pool.set_profiling(True)
        pool.kernel_times()
        for i in range(args.warmup + args.steps):
            kb.append_quantize(pool, seqs, 0, k_new, v_new, stream=stream)
            kb.decode_attention(pool, seqs, 0, q, out, cfg["scale"], stream=stream)
            torch.cuda.synchronize()
            am, an, pm, pn = pool.kernel_times()
            print(f"[rank {rank} dev {torch.cuda.current_device()}] step {i}: attn {am:.3f} ms "
                  f"append {pm:.3f} ms err {pool.device_error()} plan {pool.last_plan()}",
                  file=sys.stderr, flush=True)
        pool.set_profiling(False)
    for _ in range(args.warmup):
        kb.decode_step(pool, seqs, 0, k_new, v_new, q, out, cfg["scale"], stream=stream)
    torch.cuda.synchronize()
    barrier()
    len_before = [s.length(0) for s in seqs]
    # A step whose bytes fit in L2 would be served from it on the next step:
    # then each step is timed alone, with an L2 flush (a write of 2 x L2)
    # between steps, outside the timed pairs. Otherwise the inputs are larger
    # than L2 and the steps run back to back.
    flush = None
    if step_bytes([L + 1 for L in len_before], cfg, raw)[1] < L2_FLUSH_BYTES:
        flush = torch.zeros(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)
    n_pairs = 1 if flush is None else args.steps
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(n_pairs)]

    def timed_steps(profile):
        """K steps; with profile the library brackets each of its launches
        with CUDA events on the launching stream (per-kernel device times)."""
        pool.set_profiling(profile)
        pool.kernel_times()
        pool.kernel_count()
        torch.cuda.synchronize()
        for i in range(args.steps):
            if flush is not None:
                flush.add_(1)
            if flush is not None or i == 0:
                evs[min(i, n_pairs - 1)][0].record(stream)
            kb.decode_step(pool, seqs, 0, k_new, v_new, q, out, cfg["scale"], stream=stream)
            if flush is not None or i == args.steps - 1:
                evs[min(i, n_pairs - 1)][1].record(stream)
        torch.cuda.synchronize()
        res = (sum(a.elapsed_time(b) for a, b in evs), pool.kernel_count(), pool.kernel_times())
        pool.set_profiling(False)
        return res

    # `value`: the step as a user runs it (no per-launch events); then the
    # same number of steps again with the per-kernel events for the roofline
    # the K-step region is repeated REPEATS times, each the max over ranks;
    # `value` uses the median repetition
    # every repetition (and the profiled pass) starts from the same cache
    # lengths: the sequences are truncated back between them, outside the
    # timed region (the workload is K steps from the configured lengths)
    def rewind():
        torch.cuda.synchronize()
        for s_, L_ in zip(seqs, len_before):
            s_.truncate(L_)

    reps = []
    with ClockSampler(local_rank) as clocks:
        for _ in range(REPEATS):
            total_ms, launches, _ = timed_steps(False)
            reps.append(max_over_ranks(total_ms / args.steps))
            plan, kernels = pool.last_plan(), pool.last_kernels()
            rewind()
    barrier()
    _, _, (attn_total, attn_n, app_total, app_n) = timed_steps(True)
    rewind()
    barrier()
    attn_ms = [attn_total / max(1, attn_n)]
    app_ms = [app_total / max(1, app_n)]
    ms_step = float(np.median(reps))
    tokens_per_step = n_total
    value = tokens_per_step / (ms_step / 1e3)

    # algorithmic bytes: lengths after each step's append (the profiled pass
    # runs after the value pass, args.steps tokens further on)
    attn_bytes, step_b = 0, 0
    for i in range(args.steps):  # every repetition runs from len_before
        step_b += step_bytes([L + i + 1 for L in len_before], cfg, raw)[1]
        attn_bytes += step_bytes([L + i + 1 for L in len_before], cfg, raw)[0]
    attn_bytes /= args.steps
    step_b /= args.steps
    attn_mean_ms = float(np.mean(attn_ms))
    peak, peak_kind = measured_peak()
    achieved = attn_bytes / (attn_mean_ms / 1e3) / 1e9
    step_gbs = step_b / (ms_step / 1e3) / 1e9

    # ---- end to end through the C ABI with host buffers ----
    h_k = torch.empty(k_new.shape, dtype=tdt, pin_memory=True).copy_(k_new.cpu())
    h_v = torch.empty(v_new.shape, dtype=tdt, pin_memory=True).copy_(v_new.cpu())
    h_q = torch.empty(q.shape, dtype=tdt, pin_memory=True).copy_(q.cpu())
    h_out = torch.empty(out.shape, dtype=tdt, pin_memory=True)
    e2e_steps = max(3, args.steps // 2)
    # krill_decode_step_host: the public call for a step whose inputs and
    # output live in host memory; it overlaps the copies of one chunk of
    # layers with the kernels of its neighbours. One untimed call first (it
    # sizes the device staging), then wall-clock steps, each ending with the
    # host waiting for its output.
    kb.decode_step_host(pool, seqs, 0, h_k, h_v, h_q, h_out, cfg["scale"], layer_chunk=args.e2e_chunk,
                        stream=stream)
    torch.cuda.synchronize()
    barrier()
    # the host link as this process sees it (pinned copies of the query)
    d_probe = torch.empty_like(q)
    pe0, pe1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    link = {}
    for name, dst, src in (("h2d_gbs", d_probe, h_q), ("d2h_gbs", h_out, d_probe)):
        for _ in range(3):
            pe0.record(stream)
            dst.copy_(src, non_blocking=True)
            pe1.record(stream)
            stream.synchronize()
        link[name] = round(q.numel() * q.element_size() / (pe0.elapsed_time(pe1) / 1e3) / 1e9, 2)
    del d_probe
    e2e_ms = []
    for _ in range(e2e_steps):
        if flush is not None:
            flush.add_(1)
            torch.cuda.synchronize()
        t0 = time.perf_counter()
        kb.decode_step_host(pool, seqs, 0, h_k, h_v, h_q, h_out, cfg["scale"],
                            layer_chunk=args.e2e_chunk, stream=stream)
        stream.synchronize()
        e2e_ms.append((time.perf_counter() - t0) * 1e3)
    e2e_s = max_over_ranks(sum(e2e_ms) / 1e3 / e2e_steps)
    barrier()
    if args.diag:
        print(f"[rank {rank}] timed {total_ms / args.steps:.3f} ms/step attn {attn_ms[0]:.3f} ms "
              f"e2e {e2e_s * 1e3:.3f} ms/step err {pool.device_error()}", file=sys.stderr, flush=True)
    h2d = (h_k.numel() + h_v.numel() + h_q.numel()) * h_k.element_size()
    d2h = h_out.numel() * h_out.element_size()
    err_flag = pool.device_error()
    peers = [None] * world
    if world > 1:
        dist.all_gather_object(peers, peer)

    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline and not raw:
            threads = os.cpu_count() or 1
            v_cpu, el = cpu_baseline(cfg, lengths_all, 1, threads, min(args.cpu_layer_sample, layers))
            cpu = {"value": v_cpu, "unit": "tokens/s", "cores": threads, "kind": "port",
                   "sample": f"{n_total} seqs x {min(args.cpu_layer_sample, layers)} of {layers} layers "
                             f"x 1 step ({el:.1f} s), scaled to all layers; oracle/ C++ restatement "
                             "of QuantizedKVCache.update dataflow + SDPA"}
        clk = clocks.summary()
        line = {
            "metric": ("bf16-KV decode-attn+append tokens/s (comparison variant)" if raw
                       else "int8-KV decode-attn+append tokens/s"),
            "value": value,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_step,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16" if raw else "u8",
            "data": "synthetic",
            "config": headline_config(args, cfg, world, lengths_all, mine, raw),
            "plan": {"pieces_subblocks": plan[0], "kv_heads_per_item": plan[1], "items": plan[2],
                     "ctas": plan[3], "kernels": kernels},
            "ms_per_step_repeats": reps,
            "timing": (f"{REPEATS} repetitions of the {args.steps}-step region from the same cache "
                       "lengths (rewound between them, untimed), each the max over ranks; value and "
                       "ms_per_step from the median one (sustained load: later repetitions may run "
                       "at power-capped clocks, see clocks)"),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak,
                         "traffic": None if raw else profiled_traffic(args.config, attn_bytes),
                         "kernel": "attn_tc_kernel", "peak_kind": peak_kind,
                         "attn_ms": attn_mean_ms, "append_ms": float(np.mean(app_ms)),
                         "step_gbs": step_gbs, "algo_bytes_attn": attn_bytes,
                         "algo_bytes_step": step_b},
            "e2e": {"value": n_total / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "api": "krill_decode_step_host",
                    "layer_chunk": args.e2e_chunk, "ms_steps": [round(x, 4) for x in e2e_ms],
                    "link": link, "over_value": (n_total / e2e_s) / value,
                    "bound": ("host link: the step moves h2d + d2h bytes over PCIe each step, "
                              "the query read in place by the attention kernel")},
            "gpu_launches": launches,
            "clocks": clk,
            "prefix_peer_import": [x for x in peers if x],
            "prefill_s": t_fill,
            "device_error_flag": err_flag,
        }
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    pool.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
