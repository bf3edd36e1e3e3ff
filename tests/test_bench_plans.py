"""The planner's decision for every workload bench.py times, pinned on the
CPU with dry-run pools (device=-1: the same planning code, no kernels): the
plan and kernel instances must be the ones in tests/_bench_plans.py at every
step bench.py runs (its warm-up, value and profiled passes add up to ~50
tokens per sequence), so the GPU parity tests at those plans cover the
measured launches."""
import ctypes as C

import pytest

import bench
import krill_b200 as kb
from krill_b200 import _lib as L
from krill_b200.shard import lpt_partition
from tests._bench_plans import PLANS


def _plans(cfg, lengths, layers, window=0, steps=50):
    p = kb.KVPool(layers, cfg["hkv"], cfg["hq"], cfg["D"], num_blocks=1 << 20, group_size=cfg["G"],
                  window=window, max_append=256 if window else 0, device=-1)
    seqs = [p.create_sequence() for _ in lengths]
    arr = (C.c_uint64 * len(seqs))(*[s.handle for s in seqs])
    for s, Lq in zip(seqs, lengths):
        one = (C.c_uint64 * 1)(s.handle)
        chunk = 256 if window else Lq
        for t0 in range(0, Lq, chunk):
            L.check(L.lib.krill_append_quantize(p.handle, 1, one, 0, layers, min(chunk, Lq - t0), None,
                                                None, L.DTYPE_BF16, None))
    seen = set()
    for _ in range(steps):
        L.check(L.lib.krill_append_quantize(p.handle, len(seqs), arr, 0, layers, 1, None, None,
                                            L.DTYPE_BF16, None))
        L.check(L.lib.krill_decode_attention(p.handle, len(seqs), arr, 0, layers, None, L.DTYPE_BF16,
                                             None, L.DTYPE_BF16, 1.0, None))
        seen.add((p.last_plan(), p.last_kernels()))
    p.close()
    return seen


@pytest.mark.parametrize("key,seqs", [
    ("llama31_8b_batch32", 32), ("qwen3_30b_longctx", 16),
    ("qwen3_30b_longctx/8gpu", 2),  # configs[3]'s 16 sequences, 2 per GPU at 8 GPUs
    ("gemma_mixed_256/sliding", 256)])
def test_bench_workload_plan_is_pinned(key, seqs):
    name = key.split("/")[0]
    cfg = bench.CONFIGS[name]
    lengths_all = bench.sample_lengths(cfg, seqs)
    lengths = [lengths_all[i] for i in lpt_partition(lengths_all, 1)[0]]
    if name == "gemma_mixed_256":
        seen = _plans(cfg, lengths, cfg["layers_sliding"], window=cfg["window"])
    else:
        seen = _plans(cfg, lengths, cfg["layers"])
    assert seen == {PLANS[key]}


def test_verify_workload_uses_two_query_tiles():
    # bench.py --config next_verify4: 4 drafts x GQA 4 = 16 columns per
    # sequence, one decode item per piece with two 8-column query tiles
    cfg = bench.CONFIGS["next_verify4"]
    lengths = bench.sample_lengths(cfg, cfg["seqs"])
    layers, nq = cfg["layers"], cfg["n_query"]
    p = kb.KVPool(layers, cfg["hkv"], cfg["hq"], cfg["D"], num_blocks=1 << 20, group_size=cfg["G"],
                  device=-1)
    seqs = [p.create_sequence() for _ in lengths]
    arr = (C.c_uint64 * len(seqs))(*[s.handle for s in seqs])
    for s, Lq in zip(seqs, lengths):
        one = (C.c_uint64 * 1)(s.handle)
        L.check(L.lib.krill_append_quantize(p.handle, 1, one, 0, layers, Lq, None, None,
                                            L.DTYPE_BF16, None))
    kernels = set()
    for _ in range(3):
        L.check(L.lib.krill_append_quantize(p.handle, len(seqs), arr, 0, layers, nq, None, None,
                                            L.DTYPE_BF16, None))
        L.check(L.lib.krill_verify_attention(p.handle, len(seqs), arr, 0, layers, nq, None,
                                             L.DTYPE_BF16, None, L.DTYPE_BF16, 1.0, None))
        kernels.add(p.last_kernels())
    p.close()
    assert kernels == {"attn_tc_kernel<128,2,8,1,13,0,2>+attn_combine_kernel<128>"}, kernels
