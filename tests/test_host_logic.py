"""Host-side cache logic on a dry-run pool (device=-1): block accounting,
copy-on-write, truncate/restore semantics of QuantizedKVCache and
RotatingKVCache, the prefix cache (exact scan, LCP, LRU, isolation), forks,
and the decode-attention planner. No GPU is used; the same code runs on device
pools, where it also issues the kernels."""
import ctypes as C

import numpy as np
import pytest

import krill_b200 as kb
from krill_b200 import _lib as L


def pool(layers=2, hkv=8, hq=32, D=128, blocks=64, **kw):
    return kb.KVPool(layers, hkv, hq, D, num_blocks=blocks, device=-1, **kw)


def append(p, seqs, n_new, layer_begin=0, layer_count=None):
    lc = p.num_layers if layer_count is None else layer_count
    arr = (C.c_uint64 * len(seqs))(*[s.handle for s in seqs])
    L.check(L.lib.krill_append_quantize(p.handle, len(seqs), arr, layer_begin, lc, n_new, None, None,
                                        L.DTYPE_BF16, None))


def attend(p, seqs, layer_begin=0, layer_count=None):
    lc = p.num_layers if layer_count is None else layer_count
    arr = (C.c_uint64 * len(seqs))(*[s.handle for s in seqs])
    L.check(L.lib.krill_decode_attention(p.handle, len(seqs), arr, layer_begin, lc, None, 1, None, 2,
                                         1.0, None))
    return p.last_plan()


# ------------------------------------------------------------------ blocks
def test_append_allocates_blocks_and_tracks_lengths():
    p = pool()
    s = p.create_sequence()
    append(p, [s], 300)
    assert s.length(0) == 300 and s.length(1) == 300
    assert len(s.blocks()) == 2 and p.free_blocks == 62
    append(p, [s], 1, layer_begin=1, layer_count=1)  # per-layer update, as Gemma4Attention calls it
    assert s.length(0) == 300 and s.length(1) == 301
    append(p, [s], 212)
    assert s.length(0) == 512 and len(s.blocks()) == 3  # layer 1 at 513 needs a third block
    s.release()
    assert p.free_blocks == 64


def test_oom_is_reported_and_state_kept():
    p = pool(blocks=2)
    s = p.create_sequence()
    append(p, [s], 512)
    with pytest.raises(kb.KrillError) as e:
        append(p, [s], 1)
    assert e.value.status == L.KRILL_ERR_OOM
    assert s.length(0) == 512


def test_truncate_semantics_quantized_cache():
    """QuantizedKVCache.truncate (QuantizedKVCache.swift:135-145): n >= len
    and n < 0 are no-ops; blocks past the new length are released."""
    p = pool()
    s = p.create_sequence()
    append(p, [s], 600)
    s.truncate(700)
    assert s.length(0) == 600
    s.truncate(-3)
    assert s.length(0) == 600
    s.truncate(257)
    assert s.length(0) == 257 and len(s.blocks()) == 2
    s.truncate(0)
    assert s.length(0) == 0 and len(s.blocks()) == 0 and p.free_blocks == 64
    assert s.can_truncate(0) and not s.can_truncate(-1)


def test_memory_size_bytes():
    """memorySizeBytes (QuantizedKVCache.swift:33-42), per group."""
    p = pool(hkv=8, D=128)
    s = p.create_sequence()
    append(p, [s], 10)
    assert s.memory_size_bytes(0) == 2 * 10 * 8 * 128 + 4 * 10 * 8 * 2 * 2
    p2 = pool(hkv=8, D=128, group_size=128)
    s2 = p2.create_sequence()
    append(p2, [s2], 10)
    assert s2.memory_size_bytes(0) == 2 * 10 * 8 * 128 + 4 * 10 * 8 * 2  # the reference's formula


# ------------------------------------------------------------------ prefix cache
def test_prefix_store_lookup_fork_share_blocks():
    p = pool()
    pc = kb.PrefixCache(p, max_memory_entries=4, min_prefix_length=4)
    s = p.create_sequence()
    toks = list(range(600))
    append(p, [s], 600)
    pc.store_quantized(toks, "m-int8", s)
    assert pc.memory_count == 1
    blocks = s.blocks()
    assert [p.refcount(b) for b in blocks] == [2, 2, 2]
    hit = pc.lookup_quantized(toks, "m-int8")
    assert hit is not None and hit.prefix_length == 600 and hit.stored_length == 600
    # full hit: restore then truncate(count - 1) and re-forward the last token
    f = hit.fork(599)
    assert f.length(0) == 599 and f.blocks() == blocks
    assert [p.refcount(b) for b in blocks] == [3, 3, 3]
    free_before = p.free_blocks
    append(p, [f], 1)  # writes into the shared last block -> copy-on-write
    fb = f.blocks()
    assert fb[:2] == blocks[:2] and fb[2] != blocks[2]
    assert p.refcount(blocks[2]) == 2 and p.refcount(fb[2]) == 1
    assert p.free_blocks == free_before - 1
    hit.release()
    f.release()
    s.release()
    assert [p.refcount(b) for b in blocks] == [1, 1, 1]  # the entry still holds them
    pc.clear()
    assert pc.memory_count == 0 and p.free_blocks == 64


def test_fork_prefix_skips_prefill_and_copies_nothing():
    """Config 3 shape: a 4096-token prefix (16 full blocks) forked by many
    requests shares every block; each suffix allocates its own blocks."""
    p = pool(layers=1, blocks=200)
    pc = kb.PrefixCache(p)
    base = p.create_sequence()
    append(p, [base], 4096)
    prefix = list(range(4096))
    pc.store_quantized(prefix, "llama", base)
    reqs = []
    for r in range(64):
        hit = pc.lookup_quantized(prefix + [10_000 + r] * 256, "llama")
        # exact-key scan steps down from 4352 by 4: the 4096 prefix is found
        assert hit is None or hit.prefix_length == 4096
        hit = pc.lookup_longest_prefix_quantized(prefix + [10_000 + r] * 256, "llama")
        assert hit.prefix_length == 4096
        f = hit.fork(min(hit.prefix_length, 4352 - 1))
        hit.release()
        append(p, [f], 256)  # the unique suffix
        reqs.append(f)
    shared = base.blocks()
    assert all(r.blocks()[:16] == shared for r in reqs)
    assert p.refcount(shared[0]) == 1 + 1 + 64  # base + entry + requests
    assert p.free_blocks == 200 - 16 - 64


def test_lcp_and_min_prefix_reference_cases():
    """QuantizedPrefixCacheTests.swift:92-121: LCP of 5 with minPrefixLength 4;
    a 2-token share misses; fp16 entries are invisible (int8-only cache)."""
    p = pool()
    pc = kb.PrefixCache(p, max_memory_entries=4, min_prefix_length=4)
    s = p.create_sequence()
    append(p, [s], 8)
    pc.store_quantized([10, 11, 12, 13, 14, 15, 16, 17], "m-int8", s)
    hit = pc.lookup_longest_prefix_quantized([10, 11, 12, 13, 14, 99, 99], "m-int8")
    assert hit.prefix_length == 5 and hit.stored_length == 8
    hit.release()
    assert pc.lookup_longest_prefix_quantized([10, 11, 0, 0, 0, 0], "m-int8") is None
    assert pc.lookup_longest_prefix_quantized([10, 11, 12, 13, 14], "other-model") is None
    assert pc.lookup_longest_prefix_quantized([10, 11, 12, 13, 14], "m-int8", media_hash="img") is None
    # below minPrefixLength: nil (PrefixCacheTests.swift:29)
    assert pc.lookup_quantized([10, 11, 12], "m-int8") is None


def test_exact_scan_step_down():
    """PrefixCache.scan (PrefixCache.swift:273-308): probes the full length,
    then steps down by max(1, minPrefixLength/2) — only those lengths."""
    p = pool()
    pc = kb.PrefixCache(p, min_prefix_length=8)
    s = p.create_sequence()
    append(p, [s], 12)
    pc.store_quantized(list(range(12)), "m", s)
    assert pc.lookup_quantized(list(range(16)), "m").prefix_length == 12  # 16 -> 12
    assert pc.lookup_quantized(list(range(15)), "m") is None              # 15 -> 11 -> 7 stop
    assert pc.lookup_quantized(list(range(12)) + [99] * 4, "m").prefix_length == 12
    assert pc.lookup_quantized(list(range(11)), "m") is None


def test_lru_eviction_and_touch():
    """storeInMemory / touchEntryLocked (PrefixCache.swift:535-551)."""
    p = pool()
    pc = kb.PrefixCache(p, max_memory_entries=2, min_prefix_length=2)
    seqs = []
    for i in range(3):
        s = p.create_sequence()
        append(p, [s], 4)
        seqs.append(s)
    pc.store_quantized([1, 1, 1, 1], "m", seqs[0])
    pc.store_quantized([2, 2, 2, 2], "m", seqs[1])
    pc.lookup_quantized([1, 1, 1, 1], "m").release()   # touch entry 1
    pc.store_quantized([3, 3, 3, 3], "m", seqs[2])     # evicts entry 2 (LRU)
    assert pc.memory_count == 2
    assert pc.lookup_quantized([1, 1, 1, 1], "m") is not None
    assert pc.lookup_quantized([2, 2, 2, 2], "m") is None
    assert pc.lookup_quantized([3, 3, 3, 3], "m") is not None


def test_hit_outlives_eviction():
    p = pool()
    pc = kb.PrefixCache(p, max_memory_entries=1, min_prefix_length=2)
    a, b = p.create_sequence(), p.create_sequence()
    append(p, [a, b], 300)
    pc.store_quantized(list(range(300)), "m", a)
    hit = pc.lookup_quantized(list(range(300)), "m")
    blocks = a.blocks()
    pc.store_quantized(list(range(1, 301)), "m", b)   # evicts the first entry
    assert pc.memory_count == 1
    f = hit.fork(300)                                # still usable while held
    assert f.blocks() == blocks
    hit.release()
    assert [p.refcount(x) for x in blocks] == [2, 2]  # a + fork


def test_restore_truncate_update_lengths():
    """QuantizedPrefixCacheTests.swift:142-171: restore -> truncate(5) ->
    update(1) gives length 6 again."""
    p = pool()
    pc = kb.PrefixCache(p, min_prefix_length=4)
    s = p.create_sequence()
    append(p, [s], 6)
    pc.store_quantized(list(range(6)), "m", s)
    hit = pc.lookup_quantized(list(range(6)), "m")
    r = hit.fork(6)
    assert r.length(0) == 6
    r.truncate(5)
    assert r.length(0) == 5
    append(p, [r], 1)
    assert r.length(0) == 6


# ------------------------------------------------------------------ windowed (RotatingKVCache)
def test_rotating_retention_and_truncate_bounds():
    """RotatingKVCacheTests.swift:115-157 (window 4): after 10 single-token
    appends 4 rows are retained, positions 6..9; canTruncate(10/8/6) true,
    (5) false; truncate(8) leaves 2 retained and update resumes."""
    p = pool(layers=1, window=4, max_append=16)
    s = p.create_sequence()
    for _ in range(10):
        append(p, [s], 1)
    assert s.length(0) == 10 and s.retained(0) == 4
    assert s.can_truncate(10) and s.can_truncate(8) and s.can_truncate(6)
    assert not s.can_truncate(5)
    s.truncate(8)
    assert s.length(0) == 8 and s.retained(0) == 2
    append(p, [s], 1)
    assert s.length(0) == 9 and s.retained(0) == 3
    with pytest.raises(kb.KrillError):
        s.truncate(2)  # below the retained range: refused, not a crash


def test_rotating_restore_at_absolute_position():
    """RotatingKVCacheTests.swift:161-182: restore 3 rows at totalSeen 20."""
    p = pool(layers=1, window=4, max_append=16)
    s = p.create_sequence()
    L.check(L.lib.krill_seq_restore_quantized(p.handle, s.handle, 0, 3, 20, None, None, None, None,
                                              None, None, None))
    assert s.length(0) == 20 and s.retained(0) == 3
    assert s.can_truncate(19) and not s.can_truncate(16)
    append(p, [s], 1)
    assert s.length(0) == 21 and s.retained(0) == 4


def test_rotating_chunk_retention():
    """A chunk append keeps window-1 old rows plus the chunk
    (RotatingKVCache.update, RotatingKVCache.swift:103-113)."""
    p = pool(layers=1, window=8, max_append=16)
    s = p.create_sequence()
    for L_new, want in [(5, 5), (3, 8), (12, 19), (1, 8), (9, 16), (6, 13)]:
        append(p, [s], L_new)
        assert s.retained(0) == want
    with pytest.raises(kb.KrillError):
        append(p, [s], 17)  # above max_append


def test_windowed_ring_is_bounded():
    p = pool(layers=1, window=1024, max_append=1, blocks=64)
    s = p.create_sequence()
    append(p, [s], 1)
    for _ in range(3000):
        append(p, [s], 1)
    assert len([b for b in s.blocks() if b >= 0]) == 4  # ceil((1024 - 1 + 1) / 256)
    assert s.retained(0) == 1024


# ------------------------------------------------------------------ planner
def test_planner_adapts_to_batch_shape():
    rng = np.random.default_rng(1)
    big = pool(layers=32, blocks=2000)
    seqs = [big.create_sequence() for _ in range(32)]
    for s, n in zip(seqs, rng.integers(512, 8193, size=32)):
        append(big, [s], int(n))
    C_, HG, items, ctas = attend(big, seqs)
    assert HG == 8 and C_ >= 32 and ctas == 148 and items >= 148
    small = pool(layers=16, D=64, blocks=40)
    one = small.create_sequence()
    append(small, [one], 2048)
    C_, HG, items, ctas = attend(small, [one])
    # latency-bound: one kv head per item, the whole sequence in it (16 layers
    # x 8 heads = 128 items, no piece merged across CTAs)
    assert HG == 1 and C_ == 32 and items == 128 and ctas == 128
    # one long sequence on one layer: heads alone give 8 items, so the
    # sequence is cut into pieces of at least 8 sub-blocks to fill the GPU
    lone = pool(layers=1, D=64, blocks=200)
    s1 = lone.create_sequence()
    append(lone, [s1], 32768)
    C_, HG, items, ctas = attend(lone, [s1])
    assert HG == 1 and 8 <= C_ < 512 and 128 <= items <= 148


def test_planner_fixed_split_is_batch_invariant():
    p = pool(layers=2, split_tokens=512)
    a, b = p.create_sequence(), p.create_sequence()
    append(p, [a], 3000)
    append(p, [b], 100)
    assert attend(p, [a])[:2] == attend(p, [a, b])[:2] == (8, 8)


def _forked_batch(p, prefix, n_req, suffix):
    """n_req forks of one stored prefix, each with its own suffix appended
    (the engine's partial-hit path: restore, then prefill the suffix)."""
    pc = kb.PrefixCache(p)
    base = p.create_sequence()
    append(p, [base], prefix)
    toks = list(range(prefix))
    pc.store_quantized(toks, "m", base)
    hit = pc.lookup_quantized(toks, "m")
    forks = [hit.fork(prefix) for _ in range(n_req)]
    hit.release()
    for f in forks:
        append(p, [f], suffix)
    return pc, base, forks


def test_cascade_groups_forks_of_one_prefix():
    p = pool(layers=2, blocks=200)
    pc, base, forks = _forked_batch(p, 1024, 6, 40)
    attend(p, forks)
    groups, items, slots, ctas = p.last_cascade()
    assert groups == 1 and slots >= 1 and items >= 2 * 8 and ctas >= 1
    # an independent sequence in the batch joins no group
    lone = p.create_sequence()
    append(p, [lone], 1064)
    attend(p, forks + [lone])
    assert p.last_cascade()[0] == 1
    attend(p, [forks[0], lone])
    assert p.last_cascade() == (0, 0, 0, 0)
    pc.close()


def test_cascade_respects_switches_and_short_prefixes():
    # off, fixed split (batch-invariant results promised), windowed pools,
    # CUDA-core implementation, and a shared part below the threshold
    for kw in [dict(cascade_min_tokens=-1), dict(split_tokens=512), dict(window=2048, max_append=1024),
               dict(attn_impl=L.ATTN_CUDA_CORE)]:
        p = pool(layers=2, blocks=200, **kw)
        pc, _, forks = _forked_batch(p, 1024, 4, 10)
        attend(p, forks)
        assert p.last_cascade()[0] == 0, kw
        pc.close()
    # forks share only the prefix's full blocks: the first append into the
    # partial last block copies it (copy-on-write)
    p = pool(layers=2, blocks=200)
    pc, _, forks = _forked_batch(p, 200, 4, 10)
    attend(p, forks)
    assert p.last_cascade()[0] == 0
    pc.close()
    p = pool(layers=2, blocks=200, cascade_min_tokens=512)
    pc, _, forks = _forked_batch(p, 300, 4, 10)  # 256 shared tokens < 512
    attend(p, forks)
    assert p.last_cascade()[0] == 0
    pc.close()
    p = pool(layers=2, blocks=200)
    pc, _, forks = _forked_batch(p, 300, 4, 10)
    attend(p, forks)
    assert p.last_cascade()[0] == 1
    pc.close()


def test_cascade_shared_part_stays_below_every_length():
    """A full hit is forked at count - 1 (InferenceEngine.swift:1401-1417):
    the shared blocks then hold tokens one member never saw; the shared part
    must end before the shortest member's last token."""
    p = pool(layers=2, blocks=200, cascade_min_tokens=64)
    pc = kb.PrefixCache(p)
    base = p.create_sequence()
    append(p, [base], 300)
    toks = list(range(300))
    pc.store_quantized(toks, "m", base)
    hit = pc.lookup_quantized(toks, "m")
    a, b = hit.fork(300), hit.fork(299)
    hit.release()
    attend(p, [a, b])
    assert p.last_cascade()[0] == 1
    # the two forks share 2 blocks (512 tokens) but b holds only 299 tokens:
    # shared part = 256 (largest multiple of 64 below 298)
    attend(p, [a, b, base])
    assert p.last_cascade()[0] == 1
    pc.close()


def test_verify_attention_planning():
    """Multi-query verify: each query bounded by its own token
    (buildBatchedVerifyMask, BatchedDecode.swift:299-312); the queries must be
    in the cache; full-history pools only."""
    p = pool(layers=2, blocks=64)
    a, b = p.create_sequence(), p.create_sequence()
    append(p, [a], 500)
    append(p, [b], 3)
    arr = (C.c_uint64 * 2)(a.handle, b.handle)
    L.check(L.lib.krill_verify_attention(p.handle, 2, arr, 0, 2, 3, None, 1, None, 2, 1.0, None))
    with pytest.raises(kb.KrillError):
        L.check(L.lib.krill_verify_attention(p.handle, 2, arr, 0, 2, 4, None, 1, None, 2, 1.0, None))
    w = pool(layers=2, blocks=64, window=1024, max_append=512)
    s = w.create_sequence()
    append(w, [s], 100)
    arr1 = (C.c_uint64 * 1)(s.handle)
    st = L.lib.krill_verify_attention(w.handle, 1, arr1, 0, 2, 2, None, 1, None, 2, 1.0, None)
    assert st == L.KRILL_ERR_INVALID


def test_prefill_attention_takes_the_causal_cascade_path():
    """Many queries per sequence (chunked prefill) become causal tcgen05
    cascade items; a short verify (n_query x GQA group < 64 rows) stays on the
    per-query decode units."""
    p = pool(layers=2, blocks=64)
    s = p.create_sequence()
    append(p, [s], 1300)
    arr = (C.c_uint64 * 1)(s.handle)
    L.check(L.lib.krill_prefill_attention(p.handle, 1, arr, 0, 2, 300, None, 1, None, 2, 1.0, None))
    groups, items, slots, ctas = p.last_cascade()
    assert groups == 0 and items >= 2 * 8 * 5 and slots >= 1 and ctas >= 1  # 1200 rows -> 5 blocks
    assert p.last_plan()[2] == 0  # no decode items
    L.check(L.lib.krill_verify_attention(p.handle, 1, arr, 0, 2, 4, None, 1, None, 2, 1.0, None))
    assert p.last_cascade()[1] == 0 and p.last_plan()[2] > 0


@pytest.mark.parametrize("hq,hkv,nq,two_tiles", [
    (32, 8, 2, False),   # 8 columns: one unit, one tile
    (32, 8, 3, True),    # 12 columns: the second unit is the second tile
    (32, 8, 4, True),    # 16 columns
    (32, 8, 5, False),   # 20 columns: three units of one tile each
    (32, 4, 2, False),   # GQA 8 with 4 kv heads: no one-warp-per-head plan
    (64, 8, 2, True),    # GQA 8 with 8 kv heads: one query per tile
])
def test_verify_query_tiles(hq, hkv, nq, two_tiles):
    """Queries of one sequence share decode units as columns of the 8-column
    query tile; 9-16 columns run as two tiles of one item when the plan has
    one warp per kv head."""
    p = pool(layers=2, hkv=hkv, hq=hq, blocks=64)
    seqs = [p.create_sequence() for _ in range(3)]
    for s, n in zip(seqs, (700, 40, 300)):
        append(p, [s], n)
    arr = (C.c_uint64 * 3)(*[s.handle for s in seqs])
    L.check(L.lib.krill_verify_attention(p.handle, 3, arr, 0, 2, nq, None, 1, None, 2, 1.0, None))
    first = p.last_kernels().split("+")[0]
    assert first.startswith("attn_tc_kernel<") and first.endswith(",2>") == two_tiles, first


def test_pair_cascade_is_opt_in():
    """The CTA-pair cascade runs only under KRILL_ATTN_TENSOR_CORE_PAIR and
    only for items of more than 128 rows; a pair counts as two CTAs."""
    for impl, forks, kernel in [(L.ATTN_TENSOR_CORE, 40, "attn_shared_umma_kernel"),
                                (L.ATTN_TENSOR_CORE_PAIR, 40, "attn_shared_pair_kernel"),
                                (L.ATTN_TENSOR_CORE_PAIR, 20, "attn_shared_umma_kernel")]:
        p = pool(layers=2, blocks=400, attn_impl=impl)
        pc, _, fs = _forked_batch(p, 1024, forks, 10)
        attend(p, fs)
        groups, items, slots, ctas = p.last_cascade()
        assert groups == 1 and p.last_kernels().startswith(kernel), (impl, forks, p.last_kernels())
        if kernel == "attn_shared_pair_kernel":
            assert ctas % 2 == 0
        pc.close()
