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
    "llama32_1b_single": dict(layers=16, hq=32, hkv=8, D=64, G=64, dtype="f16", seqs=1,
                              lens=("fixed", 2048, 2048, 0), scale=1 / 8.0),
    "qwen3_30b_longctx": dict(layers=48, hq=32, hkv=4, D=128, G=64, dtype="bf16", seqs=16,
                              lens=("fixed", 32768, 32768, 3), scale=1 / math.sqrt(128)),
}
DEFAULT_CONFIG = "llama31_8b_batch32"


def algo_bytes_attn(L, hkv, D, G):
    return L * hkv * (2 * D + 8 * D // G)


def step_bytes(lengths_after, cfg):
    """Algorithmic bytes of one step (SURVEY 8(d) definition) split into the
    attention kernel's share and the whole step."""
    hkv, hq, D, G, layers = cfg["hkv"], cfg["hq"], cfg["D"], cfg["G"], cfg["layers"]
    attn = sum(algo_bytes_attn(L, hkv, D, G) for L in lengths_after) * layers
    qo = len(lengths_after) * layers * 2 * hq * D * 2
    append = len(lengths_after) * layers * (hkv * D * 4 + hkv * (2 * D + 8 * D // G))
    return attn + qo, attn + qo + append


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
                ["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.dev)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
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
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in self.rows:
            for name, val in zip(names, r[5:9]):
                if val.strip().lower() in ("active", "1"):
                    reasons.add(name)
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.rows)}


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


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


def run_reference_arm(args, cfg, rank, world):
    """--impl reference: the reference's CPU dataflow (oracle port), all host
    threads, rank 0 only."""
    if rank != 0:
        return
    import oracle
    threads = os.cpu_count() or 1
    lengths = sample_lengths(cfg, cfg["seqs"] * world)
    # bounded sample per step: every sequence, 1 of the layers
    values = []
    t_all = time.perf_counter()
    for _ in range(args.warmup):
        cpu_baseline(cfg, lengths, 1, threads, 1)
    for _ in range(args.steps):
        v, _ = cpu_baseline(cfg, lengths, 1, threads, 1)
        values.append(v)
    value = float(np.median(values))
    line = {
        "impl": "reference", "metric": "int8-KV decode-attn+append tokens/s", "value": value,
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "u8", "data": "synthetic",
        "config": {"workload": args.config, "seqs": len(lengths), "layers": cfg["layers"]},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"{len(lengths)} seqs x 1 of {cfg['layers']} layers per step, "
                                   f"scaled x{cfg['layers']}; oracle/ C++ restatement of "
                                   "QuantizedKVCache.update + SDPA (MLX CPU path unavailable)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": time.perf_counter() - t_all,
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="krill", choices=["krill", "reference"])
    ap.add_argument("--config", default=DEFAULT_CONFIG, choices=sorted(CONFIGS))
    ap.add_argument("--attn-impl", default="tc", choices=["tc", "cuda"])
    ap.add_argument("--split-tokens", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-layer-sample", type=int, default=12)
    ap.add_argument("--seqs", type=int, default=0, help="override sequences per GPU (profiling)")
    ap.add_argument("--diag", action="store_true",
                    help="per-rank, per-step kernel times and device error flags on stderr")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    cfg = dict(CONFIGS[args.config])
    if args.seqs:
        cfg["seqs"] = args.seqs

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference_arm(args, cfg, rank, world)
        return

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
        # first collective up front, so NCCL's lazy setup never overlaps our kernels
        warm = torch.ones(1, device=torch.device("cuda", local_rank))
        dist.all_reduce(warm)
        torch.cuda.synchronize()

    import krill_b200 as kb

    # ---- workload: global batch partitioned over ranks ----
    n_total = cfg["seqs"] * world
    lengths_all = sample_lengths(cfg, n_total)
    from krill_b200.shard import lpt_partition
    parts = lpt_partition(lengths_all, world)
    mine = [lengths_all[i] for i in parts[rank]]
    layers, hq, hkv, D, G = cfg["layers"], cfg["hq"], cfg["hkv"], cfg["D"], cfg["G"]
    tdt = torch.bfloat16 if cfg["dtype"] == "bf16" else torch.float16
    total_steps = args.warmup + args.steps * 2 + 2
    blocks = sum((L + total_steps + 255) // 256 for L in mine) + 4
    pool = kb.KVPool(layers, hkv, hq, D, num_blocks=blocks, group_size=G,
                     attn_impl=kb.ATTN_TENSOR_CORE if args.attn_impl == "tc" else kb.ATTN_CUDA_CORE,
                     split_tokens=args.split_tokens, device=local_rank)
    seqs = [pool.create_sequence() for _ in mine]
    dev = torch.device("cuda", local_rank)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    t_fill = time.perf_counter()
    chunk_layers = 4
    for s, L in zip(seqs, mine):
        for l0 in range(0, layers, chunk_layers):
            lc = min(chunk_layers, layers - l0)
            k = torch.randn((lc, 1, hkv, L, D), generator=gen, device=dev, dtype=torch.float32).to(tdt)
            v = torch.randn((lc, 1, hkv, L, D), generator=gen, device=dev, dtype=torch.float32).to(tdt)
            kb.append_quantize(pool, [s], l0, k, v)
            del k, v
    torch.cuda.synchronize()
    t_fill = time.perf_counter() - t_fill

    n = len(seqs)
    k_new = torch.randn((layers, n, hkv, 1, D), generator=gen, device=dev).to(tdt)
    v_new = torch.randn((layers, n, hkv, 1, D), generator=gen, device=dev).to(tdt)
    q = torch.randn((layers, n, hq, D), generator=gen, device=dev).to(tdt)
    out = torch.empty((layers, n, hq, D), dtype=tdt, device=dev)
    stream = torch.cuda.current_stream()

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
        kb.append_quantize(pool, seqs, 0, k_new, v_new, stream=stream)
        kb.decode_attention(pool, seqs, 0, q, out, cfg["scale"], stream=stream)
    torch.cuda.synchronize()
    barrier()
    len_before = [s.length(0) for s in seqs]
    # per-kernel CUDA events recorded by the library around each launch, on
    # the launching stream
    pool.set_profiling(True)
    pool.kernel_times()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        torch.cuda.synchronize()
        start.record(stream)
        for i in range(args.steps):
            kb.append_quantize(pool, seqs, 0, k_new, v_new, stream=stream)
            kb.decode_attention(pool, seqs, 0, q, out, cfg["scale"], stream=stream)
        stop.record(stream)
        torch.cuda.synchronize()
    barrier()
    total_ms = start.elapsed_time(stop)
    attn_total, attn_n, app_total, app_n = pool.kernel_times()
    pool.set_profiling(False)
    attn_ms = [attn_total / max(1, attn_n)]
    app_ms = [app_total / max(1, app_n)]
    ms_step = max_over_ranks(total_ms / args.steps)
    tokens_per_step = n_total
    value = tokens_per_step / (ms_step / 1e3)

    # algorithmic bytes: lengths after each step's append
    attn_bytes, step_b = 0, 0
    for i in range(args.steps):
        la = [L + i + 1 for L in len_before]
        a, s_ = step_bytes(la, cfg)
        attn_bytes += a
        step_b += s_
    attn_bytes /= args.steps
    step_b /= args.steps
    attn_mean_ms = float(np.mean(attn_ms))
    peak, peak_kind = measured_peak()
    achieved = attn_bytes / (attn_mean_ms / 1e3) / 1e9
    step_gbs = step_b / (total_ms / args.steps / 1e3) / 1e9

    # ---- end to end through the C ABI with host buffers ----
    h_k = torch.empty(k_new.shape, dtype=tdt, pin_memory=True).copy_(k_new.cpu())
    h_v = torch.empty(v_new.shape, dtype=tdt, pin_memory=True).copy_(v_new.cpu())
    h_q = torch.empty(q.shape, dtype=tdt, pin_memory=True).copy_(q.cpu())
    h_out = torch.empty(out.shape, dtype=tdt, pin_memory=True)
    d_k, d_v, d_q = torch.empty_like(k_new), torch.empty_like(v_new), torch.empty_like(q)
    e2e_steps = max(3, args.steps // 2)
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        d_k.copy_(h_k, non_blocking=True)
        d_v.copy_(h_v, non_blocking=True)
        d_q.copy_(h_q, non_blocking=True)
        kb.decode_step(pool, seqs, 0, d_k, d_v, d_q, out, cfg["scale"], stream=stream)
        h_out.copy_(out, non_blocking=True)
        stream.synchronize()
    e2e_s = max_over_ranks((time.perf_counter() - t0) / e2e_steps)
    barrier()
    if args.diag:
        print(f"[rank {rank}] timed {total_ms / args.steps:.3f} ms/step attn {attn_ms[0]:.3f} ms "
              f"e2e {e2e_s * 1e3:.3f} ms/step err {pool.device_error()}", file=sys.stderr, flush=True)
    h2d = (h_k.numel() + h_v.numel() + h_q.numel()) * h_k.element_size()
    d2h = h_out.numel() * h_out.element_size()
    err_flag = pool.device_error()

    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            threads = os.cpu_count() or 1
            v_cpu, el = cpu_baseline(cfg, lengths_all, 1, threads, min(args.cpu_layer_sample, layers))
            cpu = {"value": v_cpu, "unit": "tokens/s", "cores": threads, "kind": "port",
                   "sample": f"{n_total} seqs x {min(args.cpu_layer_sample, layers)} of {layers} layers "
                             f"x 1 step ({el:.1f} s), scaled to all layers; oracle/ C++ restatement "
                             "of QuantizedKVCache.update dataflow + SDPA"}
        clk = clocks.summary()
        line = {
            "metric": "int8-KV decode-attn+append tokens/s",
            "value": value,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_step,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "u8",
            "data": "synthetic",
            "config": {"workload": args.config, "layers": layers, "q_heads": hq, "kv_heads": hkv,
                       "head_dim": D, "group_size": G, "kv_in_dtype": cfg["dtype"],
                       "seqs_per_gpu": cfg["seqs"], "global_seqs": n_total,
                       "mean_len": float(np.mean(lengths_all)),
                       "l2": f"inputs larger than L2 ({step_b / 1e9:.2f} GB/step)",
                       "attn_impl": args.attn_impl, "parallelism": f"seq-partition x{world}"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak,
                         "traffic": profiled_traffic(args.config, attn_bytes),
                         "kernel": "attn_tc_kernel", "peak_kind": peak_kind,
                         "attn_ms": attn_mean_ms, "append_ms": float(np.mean(app_ms)),
                         "step_gbs": step_gbs, "algo_bytes_attn": attn_bytes,
                         "algo_bytes_step": step_b},
            "e2e": {"value": n_total / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": 2 * args.steps,
            "clocks": clk,
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
