"""The C-ABI library: loads, exports exactly what include/krill_kv.h declares,
validates arguments, and reports errors as status codes. CPU only (no kernel
is launched)."""
import ctypes as C
import os
import re

import pytest

import krill_b200 as kb
from krill_b200 import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "krill_kv.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"^\s*(?:krill_status_t|const char\*|uint64_t)\s+(krill_\w+)\s*\(", text, re.M))


def test_header_symbols_exported():
    names = declared_functions()
    assert len(names) >= 40
    for n in names:
        assert hasattr(L.lib, n), f"{n} declared in krill_kv.h but not exported"
    assert names == set(L.EXPORTED), "ctypes table and header disagree"


def test_library_has_no_torch_dependency():
    # the product library links only the CUDA runtime statically
    with open(L.LIB_PATH, "rb") as f:
        blob = f.read()
    assert b"libtorch" not in blob and b"libc10" not in blob


def test_version_and_error_string():
    assert b"sm_100a" in L.lib.krill_version()
    st = L.lib.krill_pool_create(None, -1, C.byref(C.c_void_p()))
    assert st == L.KRILL_ERR_INVALID
    assert "null" in L.last_error()


@pytest.mark.parametrize("kw,msg", [
    (dict(head_dim=96), "head_dim"),
    (dict(num_q_heads=12, num_kv_heads=8), "multiple"),
    (dict(num_q_heads=64, num_kv_heads=4), "ratio"),
    (dict(group_size=32), "group_size"),
    (dict(window=1), "window"),
    (dict(num_blocks=0), "num_blocks"),
    (dict(num_kv_heads=3, num_q_heads=6), "num_kv_heads"),
    (dict(split_tokens=100), "split_tokens"),
])
def test_pool_config_validation(kw, msg):
    args = dict(num_layers=2, num_kv_heads=8, num_q_heads=32, head_dim=128, num_blocks=8)
    args.update(kw)
    with pytest.raises(kb.KrillError) as e:
        kb.KVPool(device=-1, **args)
    assert e.value.status == L.KRILL_ERR_INVALID
    assert msg in str(e.value)


def test_block_geometry():
    p = kb.KVPool(32, 8, 32, 128, num_blocks=4, device=-1)
    # 256 tokens x (2*128 codes + 8 * 128/64 meta bytes) per (layer, head)
    assert p.block_bytes == 32 * 8 * 256 * (2 * 128 + 8 * 2)
    assert p.free_blocks == 4
    p2 = kb.KVPool(16, 8, 32, 64, num_blocks=4, device=-1)
    assert p2.block_bytes == 16 * 8 * 256 * (2 * 64 + 8)


def test_stale_handles_rejected():
    p = kb.KVPool(2, 8, 32, 128, num_blocks=8, device=-1)
    s = p.create_sequence()
    s.release()
    with pytest.raises(kb.KrillError) as e:
        s.length(0)
    assert e.value.status == L.KRILL_ERR_INVALID
    s2 = p.create_sequence()  # slot reused, new generation
    assert s2.handle != s.handle
    assert s2.length(0) == 0


def test_device_only_calls_on_host_pool():
    p = kb.KVPool(2, 8, 32, 128, num_blocks=8, device=-1)
    s = p.create_sequence()
    arr = (C.c_uint64 * 1)(s.handle)
    L.check(L.lib.krill_append_quantize(p.handle, 1, arr, 0, 2, 5, None, None, L.DTYPE_BF16, None))
    st = L.lib.krill_seq_snapshot_dequantized(p.handle, s.handle, 0, None, None, None)
    assert st == L.KRILL_ERR_NO_DEVICE
    st = L.lib.krill_decode_attention_noalloc(p.handle, 1, arr, 0, 2, None, 1, None, 1, 1.0, None)
    assert st == L.KRILL_ERR_NO_DEVICE
    buf = (C.c_uint8 * 64)()
    st = L.lib.krill_decode_step_host(p.handle, 1, arr, 0, 2, buf, buf, L.DTYPE_BF16, buf, L.DTYPE_BF16,
                                      buf, L.DTYPE_BF16, 1.0, 0, None)
    assert st == L.KRILL_ERR_NO_DEVICE


def test_argument_errors():
    p = kb.KVPool(2, 8, 32, 128, num_blocks=8, device=-1)
    s = p.create_sequence()
    arr = (C.c_uint64 * 2)(s.handle, s.handle)
    # same sequence twice in one append
    st = L.lib.krill_append_quantize(p.handle, 2, arr, 0, 1, 1, None, None, L.DTYPE_BF16, None)
    assert st == L.KRILL_ERR_INVALID and "twice" in L.last_error()
    # layer range
    st = L.lib.krill_append_quantize(p.handle, 1, arr, 1, 2, 1, None, None, L.DTYPE_BF16, None)
    assert st == L.KRILL_ERR_INVALID and "layer range" in L.last_error()
    # dtype
    st = L.lib.krill_append_quantize(p.handle, 1, arr, 0, 1, 1, None, None, L.DTYPE_F32, None)
    assert st == L.KRILL_ERR_INVALID
    # attention over an empty cache
    st = L.lib.krill_decode_attention(p.handle, 1, arr, 0, 1, None, 1, None, 2, 1.0, None)
    assert st == L.KRILL_ERR_INVALID and "empty" in L.last_error()


def test_decode_mask_matches_reference_semantics():
    """buildBatchedDecodeMask (BatchedDecode.swift:277-287): -10000 on each
    row's left pad, 0 elsewhere."""
    rows = kb.build_batched_decode_mask([3, 5, 1], s_max=5, total_len=7)
    assert rows[0] == [-10000.0, -10000.0, 0, 0, 0, 0, 0]
    assert rows[1] == [0.0] * 7
    assert rows[2] == [-10000.0] * 4 + [0.0] * 3


def test_prefix_key_matches_oracle():
    import numpy as np

    import oracle
    rng = np.random.default_rng(0)
    for n in [0, 1, 7, 100]:
        toks = [int(t) for t in rng.integers(-2**40, 2**40, size=n)]
        for media in [None, "", "abc"]:
            assert kb.prefix_key(toks, "model-x", media) == oracle.prefix_key(toks, "model-x", media)


def test_bf16_pool_geometry_and_limits():
    # raw bf16 pools: 256 tokens x (2 x D x 2 bytes) per (layer, head), no groups
    p = kb.KVPool(32, 8, 32, 128, num_blocks=4, device=-1, kv_format=kb.KV_BF16)
    assert p.block_bytes == 32 * 8 * 256 * 4 * 128
    assert p.group_size == 128
    s = p.create_sequence()
    arr = (C.c_uint64 * 1)(s.handle)
    st = L.lib.krill_append_quantize(p.handle, 1, arr, 0, 1, 1, None, None, L.DTYPE_F16, None)
    assert st == L.KRILL_ERR_INVALID and "BF16" in L.last_error()
    L.check(L.lib.krill_append_quantize(p.handle, 1, arr, 0, 32, 3, None, None, L.DTYPE_BF16, None))
    st = L.lib.krill_decode_attention(p.handle, 1, arr, 0, 1, None, L.DTYPE_F16, None, 2, 1.0, None)
    assert st == L.KRILL_ERR_INVALID and "BF16 q" in L.last_error()
    for kw in [dict(head_dim=256), dict(attn_impl=L.ATTN_CUDA_CORE), dict(kv_format=7)]:
        args = dict(num_layers=2, num_kv_heads=8, num_q_heads=32, head_dim=128, num_blocks=4,
                    kv_format=kb.KV_BF16)
        args.update(kw)
        with pytest.raises(kb.KrillError):
            kb.KVPool(device=-1, **args)


def test_disk_tier_needs_a_device_pool(tmp_path):
    p = kb.KVPool(2, 8, 32, 128, num_blocks=4, device=-1)
    pc = kb.PrefixCache(p)
    pc.set_disk(str(tmp_path), 0)  # budget 0 = disabled: always accepted
    assert pc.disk_count == 0
    with pytest.raises(kb.KrillError) as e:
        pc.set_disk(str(tmp_path), -1)
    assert e.value.status == L.KRILL_ERR_NO_DEVICE
    pc.wait_for_disk_writes()
    pc.close()


def test_entry_descriptor_and_ipc_need_devices():
    p = kb.KVPool(2, 8, 32, 128, num_blocks=8, device=-1)
    pc = kb.PrefixCache(p)
    s = p.create_sequence()
    arr = (C.c_uint64 * 1)(s.handle)
    L.check(L.lib.krill_append_quantize(p.handle, 1, arr, 0, 2, 300, None, None, L.DTYPE_BF16, None))
    pc.store_quantized(list(range(300)), "m", s)
    hit = pc.lookup_quantized(list(range(300)), "m")
    desc = pc.describe(hit)
    assert desc[:4] == b"KKV1" and len(desc) > 300 * 8
    with pytest.raises(kb.KrillError) as e:
        p.ipc_handle()
    assert e.value.status == L.KRILL_ERR_NO_DEVICE
    with pytest.raises(kb.KrillError) as e:
        pc.import_entry(b"\0" * 64, desc)
    assert e.value.status == L.KRILL_ERR_NO_DEVICE
    hit.release()
    pc.close()


def test_pool_wait_limit_is_validated():
    """krill_pool_cfg.wait_timeout_us: 0 takes the default, negative is refused."""
    import krill_b200 as kb
    kb.KVPool(2, 8, 32, 128, num_blocks=4, device=-1, wait_timeout_us=0).close()
    kb.KVPool(2, 8, 32, 128, num_blocks=4, device=-1, wait_timeout_us=1000).close()
    with pytest.raises(L.KrillError) as ei:
        kb.KVPool(2, 8, 32, 128, num_blocks=4, device=-1, wait_timeout_us=-1)
    assert ei.value.status == L.KRILL_ERR_INVALID
