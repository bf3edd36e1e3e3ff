"""Prefix-cache disk tier (PrefixCache.swift:496-501 naming, :553-581 load,
:583-648 write + budget, :650-695 LRU eviction): files are written behind the
caller in the reference's safetensors layout, survive a restart (a new pool
and cache on the same directory hit them), serve full-match hits only, obey
the byte budget by recency, and a file in the reference's own layout loads."""
import math
import os
import time

import numpy as np
import pytest

import oracle
from tests import _safetensors as st
from tests._data import BF16, F16, kv_values, to_bits

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

import krill_b200 as kb  # noqa: E402
from tests._gpu import dev_bits, host_bits, prefill  # noqa: E402

D, HQ, HKV, LAYERS = 128, 32, 8, 2


def fname(tokens, model):
    return f"{kb.prefix_key(tokens, model):016x}.q8.safetensors"


def attn(pool, seq, q):
    out = torch.empty((LAYERS, 1, HQ, D), dtype=torch.float32, device="cuda")
    kb.decode_attention(pool, [seq], 0, q, out, 1 / math.sqrt(D))
    torch.cuda.synchronize()
    return out


def test_disk_write_layout_and_restart_hit(tmp_path):
    rng = np.random.default_rng(0)
    pool = kb.KVPool(LAYERS, HKV, HQ, D, num_blocks=32)
    pc = kb.PrefixCache(pool, cache_dir=str(tmp_path), disk_budget_bytes=-1)
    base = pool.create_sequence()
    k = to_bits(kv_values(rng, (LAYERS, HKV, 600, D)), BF16)
    v = to_bits(kv_values(rng, (LAYERS, HKV, 600, D)), BF16)
    prefill(pool, base, k, v, BF16)
    toks = [int(t) for t in rng.integers(0, 50000, size=600)]
    pc.store_quantized(toks, "llama", base)
    pc.wait_for_disk_writes()
    assert pc.disk_count == 1
    path = os.path.join(str(tmp_path), fname(toks, "llama"))
    tensors, header = st.read(path)
    assert len(tensors) == 6 * LAYERS
    for layer in range(LAYERS):
        snap = base.quantized_snapshot(layer)
        exp = {"qk": ("U8", snap.keys.cpu().numpy()), "qv": ("U8", snap.values.cpu().numpy()),
               "ks": ("F16", host_bits(snap.key_scales)), "kz": ("F16", host_bits(snap.key_zeros)),
               "vs": ("F16", host_bits(snap.value_scales)), "vz": ("F16", host_bits(snap.value_zeros))}
        for suffix, (dt, arr) in exp.items():
            got_dt, got = tensors[f"layer_{layer}_{suffix}"]
            assert got_dt == dt and got.shape == (1,) + arr.shape
            np.testing.assert_array_equal(got[0], arr)
    q = dev_bits(to_bits(kv_values(rng, (LAYERS, 1, HQ, D)), BF16), BF16)
    want = attn(pool, base, q)
    pc.close()
    pool.close()

    # "restart": a new pool and cache on the same directory
    pool2 = kb.KVPool(LAYERS, HKV, HQ, D, num_blocks=32)
    pc2 = kb.PrefixCache(pool2, cache_dir=str(tmp_path), disk_budget_bytes=-1)
    assert pc2.memory_count == 0
    # the scan steps down by max(1, minPrefixLength / 2) = 4 from 604: 600 is probed
    hit = pc2.lookup_quantized(toks + [1, 2, 3, 4], "llama")
    assert hit is not None and hit.prefix_length == 600 and pc2.memory_count == 1
    f = hit.fork(600)
    hit.release()
    assert torch.equal(attn(pool2, f, q), want)
    # disk-loaded entries carry no tokens: no longest-prefix match
    assert pc2.lookup_longest_prefix_quantized(toks[:300] + [7] * 20, "llama") is None
    # another model id never hits
    assert pc2.lookup_quantized(toks, "other") is None
    pc2.clear()
    assert pc2.disk_count == 0 and not os.path.exists(os.path.join(str(tmp_path), fname(toks, "llama")))
    pc2.close()
    pool2.close()


def test_disk_budget_evicts_least_recent(tmp_path):
    """Budget of 2.5 entries: after the third file the oldest is evicted
    (down to 90 %); a disk hit refreshes an entry's recency, so entry 1, read
    back from disk, outlives the newer entry 2 when entry 3 is written."""
    rng = np.random.default_rng(1)
    pool = kb.KVPool(LAYERS, HKV, HQ, D, num_blocks=64)
    one = LAYERS * HKV * 256 * (2 * D + 8 * D // 64)  # data bytes of a 256-token entry
    # one memory slot, so earlier entries are served from disk
    pc = kb.PrefixCache(pool, max_memory_entries=1, cache_dir=str(tmp_path),
                        disk_budget_bytes=int(2.5 * one))
    prompts = [[i * 1000 + t for t in range(256)] for i in range(4)]

    def store(i):
        s = pool.create_sequence()
        k = to_bits(kv_values(rng, (LAYERS, HKV, 256, D)), BF16)
        prefill(pool, s, k, k, BF16)
        pc.store_quantized(prompts[i], "m", s)
        pc.wait_for_disk_writes()
        s.release()
        time.sleep(0.05)  # distinct modification times

    for i in range(3):
        store(i)
    files = set(os.listdir(str(tmp_path)))
    assert files == {fname(prompts[1], "m"), fname(prompts[2], "m")}
    hit = pc.lookup_quantized(prompts[1], "m")  # memory holds entry 2: a disk hit
    assert hit is not None and hit.prefix_length == 256
    hit.release()
    time.sleep(0.05)
    store(3)
    files = set(os.listdir(str(tmp_path)))
    assert files == {fname(prompts[1], "m"), fname(prompts[3], "m")}
    pc.close()
    pool.close()


@pytest.mark.parametrize("dtype", [F16, BF16])
def test_reference_layout_file_loads(tmp_path, dtype):
    """A file in the reference's own layout (one scale per (token, head):
    G = D, F16 [1, H, S, 1] scales; MLX writes a "__metadata__" block) is
    hydrated into a G = D pool and serves a full hit with the file's bytes."""
    rng = np.random.default_rng(2)
    S = 300
    toks = list(range(S))
    tensors = {}
    for layer in range(LAYERS):
        k = to_bits(kv_values(rng, (HKV, S, D)), dtype)
        v = to_bits(kv_values(rng, (HKV, S, D)), dtype)
        ck, sk, zk = oracle.quantize(k, dtype, D)
        cv, sv, zv = oracle.quantize(v, dtype, D)
        for suffix, dt, arr in [("qk", "U8", ck), ("qv", "U8", cv), ("ks", "F16", sk), ("kz", "F16", zk),
                                ("vs", "F16", sv), ("vz", "F16", zv)]:
            tensors[f"layer_{layer}_{suffix}"] = (dt, arr.reshape((1,) + arr.shape))
    st.write(os.path.join(str(tmp_path), fname(toks, "gemma")), tensors, metadata={"format": "mlx"})
    pool = kb.KVPool(LAYERS, HKV, HQ, D, num_blocks=16, group_size=D)
    pc = kb.PrefixCache(pool, cache_dir=str(tmp_path), disk_budget_bytes=-1)
    assert pc.disk_count == 1
    hit = pc.lookup_quantized(toks, "gemma")
    assert hit is not None and hit.prefix_length == S
    f = hit.fork(S)
    hit.release()
    for layer in range(LAYERS):
        snap = f.quantized_snapshot(layer)
        np.testing.assert_array_equal(snap.keys.cpu().numpy(), tensors[f"layer_{layer}_qk"][1][0])
        np.testing.assert_array_equal(host_bits(snap.value_zeros), tensors[f"layer_{layer}_vz"][1][0])
    # a file whose shapes do not fit the pool is a miss, not an error
    pool64 = kb.KVPool(LAYERS, HKV, HQ, D, num_blocks=16, group_size=64)
    pc64 = kb.PrefixCache(pool64, cache_dir=str(tmp_path), disk_budget_bytes=-1)
    assert pc64.lookup_quantized(toks, "gemma") is None
    pc64.close()
    pool64.close()
    pc.close()
    pool.close()
