"""Python mirror of Krill's cache API over the C ABI.

Names follow the reference (Sources/KrillCache/*.swift,
Sources/KrillEngine/BatchedDecode.swift) so that tests read like the
reference's own: ``QuantizedKVCache`` (one layer of one request),
``PrefixCache``, ``make_quantized_kv_caches``,
``stack_caches_left_padded_quantized``, ``build_batched_decode_mask`` and
``scatter_back``. The hot path is ``decode_step`` / ``decode_attention`` /
``append_quantize``, which run whole batches through the sm_100a kernels.

PyTorch is used only to hold device buffers and streams; every computation is
a call into libkrill_kv.so.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional, Sequence

from . import _lib as L
from ._lib import check

try:  # torch is plumbing: device buffers and the current stream
    import torch
except ImportError:  # pragma: no cover - host-only use
    torch = None

_TORCH_DT = {}
if torch is not None:
    _TORCH_DT = {torch.float16: L.DTYPE_F16, torch.bfloat16: L.DTYPE_BF16, torch.float32: L.DTYPE_F32,
                 torch.uint8: L.DTYPE_U8}


def _dt(t) -> int:
    return _TORCH_DT[t.dtype]


def _ptr(t) -> Optional[int]:
    if t is None:
        return None
    if not t.is_contiguous():
        raise ValueError("tensors passed to the C ABI must be contiguous")
    return t.data_ptr()


def _stream(stream) -> Optional[int]:
    if stream is not None:
        return stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)
    if torch is not None and torch.cuda.is_available() and torch.cuda.is_initialized():
        return torch.cuda.current_stream().cuda_stream
    return None


def _seq_array(seqs: Sequence["Sequence_"]):
    arr = (C.c_uint64 * len(seqs))(*[s.handle for s in seqs])
    return arr


class KVPool:
    """One device-resident block pool for a layer group (256-token blocks,
    int8 codes + fp16 scale/zero per group). ``device=-1`` makes a host-only
    pool (accounting and prefix logic only)."""

    def __init__(self, num_layers: int, num_kv_heads: int, num_q_heads: int, head_dim: int,
                 num_blocks: int, group_size: int = 64, window: int = 0, max_append: int = 0,
                 quant_variant: int = L.QUANT_F32, attn_impl: int = L.ATTN_TENSOR_CORE,
                 split_tokens: int = 0, cascade_min_tokens: int = 0, kv_format: int = L.KV_INT8,
                 device: int = 0, wait_timeout_us: int = 0):
        cfg = L.PoolCfg(num_layers, num_kv_heads, num_q_heads, head_dim, group_size, window,
                        max_append, quant_variant, attn_impl, split_tokens, cascade_min_tokens,
                        kv_format, num_blocks, wait_timeout_us)
        h = C.c_void_p()
        check(L.lib.krill_pool_create(C.byref(cfg), device, C.byref(h)))
        self.handle = h
        self.cfg = cfg
        self.device = device
        self.num_layers, self.num_kv_heads, self.num_q_heads = num_layers, num_kv_heads, num_q_heads
        self.head_dim, self.window, self.kv_format = head_dim, window, kv_format
        self.group_size = head_dim if kv_format == L.KV_BF16 else group_size
        self.num_groups = head_dim // self.group_size

    def close(self):
        if self.handle:
            check(L.lib.krill_pool_destroy(self.handle))
            self.handle = None

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass

    @property
    def block_bytes(self) -> int:
        v = C.c_int64()
        check(L.lib.krill_pool_block_bytes(self.handle, C.byref(v)))
        return v.value

    @property
    def free_blocks(self) -> int:
        v = C.c_int64()
        check(L.lib.krill_pool_free_blocks(self.handle, C.byref(v)))
        return v.value

    def refcount(self, block: int) -> int:
        v = C.c_int32()
        check(L.lib.krill_pool_block_refcount(self.handle, block, C.byref(v)))
        return v.value

    def device_error(self) -> int:
        v = C.c_int32()
        check(L.lib.krill_pool_device_error(self.handle, C.byref(v)))
        return v.value

    def test_stall(self, enable: bool = True):
        """Testing only: make the next decode launches' bounded wait run out
        (krill_pool_test_stall)."""
        check(L.lib.krill_pool_test_stall(self.handle, 1 if enable else 0))

    def set_profiling(self, enable: bool = True):
        check(L.lib.krill_pool_set_profiling(self.handle, 1 if enable else 0))

    def kernel_times(self):
        """(attention ms, attention launches, append ms, append launches)
        accumulated since the last call (profiling must be enabled)."""
        am, an, pm, pn = C.c_double(), C.c_int32(), C.c_double(), C.c_int32()
        check(L.lib.krill_pool_kernel_times(self.handle, C.byref(am), C.byref(an), C.byref(pm),
                                            C.byref(pn)))
        return am.value, an.value, pm.value, pn.value

    def kernel_count(self) -> int:
        """Device kernels this pool launched since the previous call."""
        v = C.c_int64()
        check(L.lib.krill_pool_kernel_count(self.handle, C.byref(v)))
        return v.value

    def last_plan(self):
        """(piece sub-blocks, kv heads per item, items, CTAs) of the last
        decode-attention launch."""
        c, hg, n, g = C.c_int32(), C.c_int32(), C.c_int64(), C.c_int32()
        check(L.lib.krill_pool_last_plan(self.handle, C.byref(c), C.byref(hg), C.byref(n), C.byref(g)))
        return c.value, hg.value, n.value, g.value

    def last_kernels(self) -> str:
        """Kernel instances of the last decode-attention launch, joined by '+'
        (e.g. 'attn_tc_kernel<128,2,8,1,13,0>+attn_combine_kernel<128>')."""
        buf = C.create_string_buffer(192)
        check(L.lib.krill_pool_last_kernels(self.handle, buf, len(buf)))
        return buf.value.decode()

    def ipc_handle(self) -> bytes:
        """This pool's CUDA IPC handle (64 bytes) for krill_prefix_import."""
        buf = C.create_string_buffer(64)
        check(L.lib.krill_pool_ipc_handle(self.handle, buf))
        return buf.raw

    def last_cascade(self):
        """(sequence groups attended together, cascade items, prefix record
        slots per member, cascade CTAs) of the last decode-attention launch."""
        g, n, s, c = C.c_int32(), C.c_int64(), C.c_int32(), C.c_int32()
        check(L.lib.krill_pool_last_cascade(self.handle, C.byref(g), C.byref(n), C.byref(s), C.byref(c)))
        return g.value, n.value, s.value, c.value

    def create_sequence(self) -> "Sequence_":
        h = C.c_uint64()
        check(L.lib.krill_seq_create(self.handle, C.byref(h)))
        return Sequence_(self, h.value)


class Sequence_:
    """One request's per-layer caches (the reference's ``[QuantizedKVCache]``
    for one row), backed by a shared block table."""

    def __init__(self, pool: KVPool, handle: int):
        self.pool = pool
        self.handle = handle

    def release(self):
        check(L.lib.krill_seq_release(self.pool.handle, self.handle))

    def reset(self):
        check(L.lib.krill_seq_reset(self.pool.handle, self.handle))

    def length(self, layer: int = 0) -> int:
        v = C.c_int64()
        check(L.lib.krill_seq_length(self.pool.handle, self.handle, layer, C.byref(v)))
        return v.value

    def retained(self, layer: int = 0) -> int:
        v = C.c_int64()
        check(L.lib.krill_seq_retained(self.pool.handle, self.handle, layer, C.byref(v)))
        return v.value

    def truncate(self, n: int):
        check(L.lib.krill_seq_truncate(self.pool.handle, self.handle, n))

    def can_truncate(self, n: int) -> bool:
        v = C.c_int32()
        check(L.lib.krill_seq_can_truncate(self.pool.handle, self.handle, n, C.byref(v)))
        return bool(v.value)

    def blocks(self) -> list:
        n = C.c_int32()
        check(L.lib.krill_seq_blocks(self.pool.handle, self.handle, None, 0, C.byref(n)))
        ids = (C.c_int32 * max(1, n.value))()
        check(L.lib.krill_seq_blocks(self.pool.handle, self.handle, ids, n.value, C.byref(n)))
        return list(ids[: n.value])

    def memory_size_bytes(self, layer: int = 0) -> int:
        v = C.c_int64()
        check(L.lib.krill_seq_memory_bytes(self.pool.handle, self.handle, layer, C.byref(v)))
        return v.value

    def layer(self, i: int) -> "QuantizedKVCache":
        return QuantizedKVCache(self, i)

    # -- snapshots ---------------------------------------------------------
    def quantized_snapshot(self, layer: int, stream=None) -> Optional["QuantizedKVSnapshot"]:
        S = self.retained(layer)
        if S == 0:
            return None
        p = self.pool
        dev = torch.device("cuda", p.device)
        keys = torch.empty((p.num_kv_heads, S, p.head_dim), dtype=torch.uint8, device=dev)
        values = torch.empty_like(keys)
        meta = [torch.empty((p.num_kv_heads, S, p.num_groups), dtype=torch.float16, device=dev)
                for _ in range(4)]
        check(L.lib.krill_seq_snapshot_quantized(p.handle, self.handle, layer, _ptr(keys), _ptr(values),
                                                 *[_ptr(m) for m in meta], _stream(stream)))
        return QuantizedKVSnapshot(keys, values, *meta)

    def snapshot(self, layer: int, stream=None):
        """Dequantized fp16 (keys, values) [Hkv, S, D], bit-exact with the
        reference's dequantize (QuantizedKVCache.swift:200-204)."""
        S = self.retained(layer)
        if S == 0:
            return None
        p = self.pool
        dev = torch.device("cuda", p.device)
        k = torch.empty((p.num_kv_heads, S, p.head_dim), dtype=torch.float16, device=dev)
        v = torch.empty_like(k)
        check(L.lib.krill_seq_snapshot_dequantized(p.handle, self.handle, layer, _ptr(k), _ptr(v),
                                                   _stream(stream)))
        return k, v

    def restore_quantized(self, layer: int, snap: "QuantizedKVSnapshot", total_seen: Optional[int] = None,
                          stream=None):
        rows = snap.keys.shape[-2]
        ts = rows if total_seen is None else total_seen
        check(L.lib.krill_seq_restore_quantized(
            self.pool.handle, self.handle, layer, rows, ts, _ptr(snap.keys), _ptr(snap.values),
            _ptr(snap.key_scales), _ptr(snap.key_zeros), _ptr(snap.value_scales),
            _ptr(snap.value_zeros), _stream(stream)))


@dataclass
class QuantizedKVSnapshot:
    """The six per-layer tensors (QuantizedKVCache.swift:150-157): u8 codes
    [Hkv, S, D] and fp16 scale/zero [Hkv, S, D/G]."""
    keys: "torch.Tensor"
    values: "torch.Tensor"
    key_scales: "torch.Tensor"
    key_zeros: "torch.Tensor"
    value_scales: "torch.Tensor"
    value_zeros: "torch.Tensor"

    @property
    def sequence_length(self) -> int:
        return self.keys.shape[-2]


class QuantizedKVCache:
    """One layer of one request: mirror of QuantizedKVCache
    (Sources/KrillCache/QuantizedKVCache.swift:17). ``update`` appends through
    the fused quantize kernel and, like the reference, returns the full
    dequantized K/V (a gather; the hot path uses ``decode_attention``)."""

    def __init__(self, seq: Sequence_, layer: int):
        self.seq = seq
        self.layer_index = layer

    @property
    def sequence_length(self) -> int:
        return self.seq.length(self.layer_index)

    @property
    def memory_size_bytes(self) -> int:
        return self.seq.memory_size_bytes(self.layer_index)

    def update(self, keys, values, stream=None):
        """keys/values: [Hkv, L_new, D] (or [1, Hkv, L_new, D]) f16/bf16."""
        k = keys.reshape(keys.shape[-3:]).contiguous()
        v = values.reshape(values.shape[-3:]).contiguous()
        append_quantize(self.seq.pool, [self.seq], self.layer_index, k, v, stream=stream)
        return self.seq.snapshot(self.layer_index, stream=stream)

    def snapshot(self, stream=None):
        return self.seq.snapshot(self.layer_index, stream=stream)

    def quantized_snapshot(self, stream=None):
        return self.seq.quantized_snapshot(self.layer_index, stream=stream)

    def restore_quantized(self, snap: QuantizedKVSnapshot, stream=None):
        self.seq.restore_quantized(self.layer_index, snap, stream=stream)

    def truncate(self, to: int):
        self.seq.truncate(to)

    def reset(self):
        self.seq.reset()


def make_quantized_kv_caches(pool: KVPool, num_layers: Optional[int] = None):
    """makeQuantizedKVCaches(numLayers:) (QuantizedKVCache.swift:208): the
    per-layer caches of one new request."""
    seq = pool.create_sequence()
    n = pool.num_layers if num_layers is None else num_layers
    return [seq.layer(i) for i in range(n)]


# ---------------------------------------------------------------- hot path
def append_quantize(pool: KVPool, seqs, layer_begin: int, k_new, v_new, stream=None, rope=None):
    """Quantize and append. k_new/v_new: [layer_count, n_seqs, Hkv, n_new, D]
    (a 3-D [Hkv, n_new, D] tensor is one layer of one sequence). ``rope`` =
    (cos, sin) f32 device tables [rows][D/2]: rotate the new K at each token's
    position first (fused RoPE + quantize + append)."""
    if k_new.dim() == 3:
        k_new = k_new.unsqueeze(0).unsqueeze(0)
        v_new = v_new.unsqueeze(0).unsqueeze(0)
    lc, ns, _, n_new, _ = k_new.shape
    assert ns == len(seqs)
    arr = _seq_array(seqs)
    if rope is None:
        check(L.lib.krill_append_quantize(pool.handle, ns, arr, layer_begin, lc, n_new, _ptr(k_new),
                                          _ptr(v_new), _dt(k_new), _stream(stream)))
        return
    cos, sin = rope
    assert cos.shape == sin.shape and cos.dim() == 2 and cos.dtype == torch.float32
    check(L.lib.krill_append_quantize_rope(pool.handle, ns, arr, layer_begin, lc, n_new, _ptr(k_new),
                                           _ptr(v_new), _dt(k_new), _ptr(cos), _ptr(sin),
                                           cos.shape[0], _stream(stream)))


def verify_attention(pool: KVPool, seqs, layer_begin: int, q, out, scale: float, stream=None):
    """Multi-query verify attention (buildBatchedVerifyMask semantics): q/out
    [layer_count, n_seqs, n_query, Hq, D]; the last n_query cached tokens of
    each sequence are the queries, each seeing the cache up to its own token."""
    lc, ns, nq = q.shape[0], q.shape[1], q.shape[2]
    assert ns == len(seqs)
    arr = _seq_array(seqs)
    check(L.lib.krill_verify_attention(pool.handle, ns, arr, layer_begin, lc, nq, _ptr(q), _dt(q),
                                       _ptr(out), _dt(out), scale, _stream(stream)))
    return out


def prefill_attention(pool: KVPool, seqs, layer_begin: int, q, out, scale: float, stream=None):
    """Chunked-prefill attention (InferenceEngine.swift:3122-3147): the chunk's
    K/V are already appended; q/out [layer_count, n_seqs, chunk, Hq, D]."""
    lc, ns, nq = q.shape[0], q.shape[1], q.shape[2]
    assert ns == len(seqs)
    arr = _seq_array(seqs)
    check(L.lib.krill_prefill_attention(pool.handle, ns, arr, layer_begin, lc, nq, _ptr(q), _dt(q),
                                        _ptr(out), _dt(out), scale, _stream(stream)))
    return out


def decode_attention(pool: KVPool, seqs, layer_begin: int, q, out, scale: float, stream=None):
    """q/out: [layer_count, n_seqs, Hq, D]."""
    lc, ns = q.shape[0], q.shape[1]
    assert ns == len(seqs)
    arr = _seq_array(seqs)
    check(L.lib.krill_decode_attention(pool.handle, ns, arr, layer_begin, lc, _ptr(q), _dt(q),
                                       _ptr(out), _dt(out), scale, _stream(stream)))
    return out


def decode_step(pool: KVPool, seqs, layer_begin: int, k_new, v_new, q, out, scale: float, stream=None):
    """Append one token per (layer, seq) and attend. k_new/v_new:
    [layer_count, n_seqs, Hkv, 1, D]; q/out: [layer_count, n_seqs, Hq, D]."""
    lc, ns = q.shape[0], q.shape[1]
    arr = _seq_array(seqs)
    check(L.lib.krill_decode_step(pool.handle, ns, arr, layer_begin, lc, _ptr(k_new), _ptr(v_new),
                                  _dt(k_new), _ptr(q), _dt(q), _ptr(out), _dt(out), scale,
                                  _stream(stream)))
    return out


def decode_step_host(pool: KVPool, seqs, layer_begin: int, k_new, v_new, q, out, scale: float,
                     layer_chunk: int = 0, stream=None):
    """decode_step with CPU tensors (page-locked for overlapped copies): the
    transfers in and out run on their own streams, a chunk of layers ahead of
    and behind the kernels. `out` is complete once `stream` has finished."""
    for t, name in ((k_new, "k_new"), (v_new, "v_new"), (q, "q"), (out, "out")):
        if t.is_cuda or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous host tensor")
    lc, ns = q.shape[0], q.shape[1]
    arr = _seq_array(seqs)
    check(L.lib.krill_decode_step_host(pool.handle, ns, arr, layer_begin, lc, _ptr(k_new), _ptr(v_new),
                                       _dt(k_new), _ptr(q), _dt(q), _ptr(out), _dt(out), scale,
                                       layer_chunk, _stream(stream)))
    return out


# ---------------------------------------------------------------- batch glue
def stack_caches_left_padded_quantized(pool: KVPool, seqs, layer: int, s_max: Optional[int] = None,
                                       stream=None) -> QuantizedKVSnapshot:
    """stackCachesLeftPaddedQuantized (BatchedDecode.swift:96-151) for one layer."""
    lens = [s.retained(layer) for s in seqs]
    sm = max(lens) if s_max is None else s_max
    dev = torch.device("cuda", pool.device)
    R, H, D, NG = len(seqs), pool.num_kv_heads, pool.head_dim, pool.num_groups
    keys = torch.empty((R, H, sm, D), dtype=torch.uint8, device=dev)
    values = torch.empty_like(keys)
    meta = [torch.empty((R, H, sm, NG), dtype=torch.float16, device=dev) for _ in range(4)]
    arr = _seq_array(seqs)
    check(L.lib.krill_stack_left_padded(pool.handle, R, arr, layer, sm, _ptr(keys), _ptr(values),
                                        *[_ptr(m) for m in meta], _stream(stream)))
    return QuantizedKVSnapshot(keys, values, *meta)


def scatter_back(pool: KVPool, seqs, layer: int, stacked: QuantizedKVSnapshot, base_lens, s_max: int,
                 steps: int, stream=None):
    """ContinuousBatcher.scatterBack int8 branch (ContinuousBatcher.swift:763-773)."""
    arr = _seq_array(seqs)
    bl = (C.c_int64 * len(seqs))(*base_lens)
    check(L.lib.krill_scatter_back(pool.handle, len(seqs), arr, layer, bl, s_max, steps,
                                   _ptr(stacked.keys), _ptr(stacked.values), _ptr(stacked.key_scales),
                                   _ptr(stacked.key_zeros), _ptr(stacked.value_scales),
                                   _ptr(stacked.value_zeros), _stream(stream)))


def build_batched_decode_mask(lengths, s_max: int, total_len: int):
    """buildBatchedDecodeMask (BatchedDecode.swift:277-287) -> list of rows."""
    n = len(lengths)
    la = (C.c_int64 * max(1, n))(*lengths)
    out = (C.c_float * max(1, n * total_len))()
    check(L.lib.krill_build_decode_mask(la, n, s_max, total_len, out))
    return [list(out[r * total_len:(r + 1) * total_len]) for r in range(n)]


# ---------------------------------------------------------------- prefix cache
def _enc(s: Optional[str]):
    return None if s is None else s.encode("utf-8")


def _tok_array(tokens):
    return (C.c_int64 * max(1, len(tokens)))(*tokens)


@dataclass
class QuantizedPrefixCacheHit:
    """QuantizedPrefixCacheHit (PrefixCache.swift:463-466): holds a reference
    on the entry until ``release``."""
    cache: "PrefixCache"
    entry: C.c_void_p
    prefix_length: int

    @property
    def stored_length(self) -> int:
        v = C.c_int64()
        check(L.lib.krill_prefix_entry_length(self.entry, C.byref(v)))
        return v.value

    def fork(self, keep: int) -> Sequence_:
        """Restore + truncate(to: keep) without copying: a new sequence sharing
        the entry's blocks (InferenceEngine.swift:1305-1320, 1401-1417)."""
        h = C.c_uint64()
        check(L.lib.krill_seq_fork_prefix(self.cache.handle, self.entry, keep, C.byref(h)))
        return Sequence_(self.cache.pool, h.value)

    def release(self):
        if self.entry:
            check(L.lib.krill_prefix_entry_release(self.cache.handle, self.entry))
            self.entry = None


class PrefixCache:
    """PrefixCache (PrefixCache.swift:15) over one pool; int8 entries only.

    ``cache_dir`` + ``disk_budget_bytes`` enable the persistent tier
    (PrefixCache.swift:496-695): 0 disables it (the default here; the
    reference defaults to 2 GB under ~/.krill/cache), a negative budget is
    unbounded."""

    def __init__(self, pool: KVPool, max_memory_entries: int = 8, min_prefix_length: int = 8,
                 cache_dir: Optional[str] = None, disk_budget_bytes: int = 0):
        h = C.c_void_p()
        check(L.lib.krill_prefix_create(pool.handle, max_memory_entries, min_prefix_length, C.byref(h)))
        self.handle = h
        self.pool = pool
        if cache_dir is not None and disk_budget_bytes != 0:
            self.set_disk(cache_dir, disk_budget_bytes)

    def set_disk(self, cache_dir: str, budget_bytes: int):
        check(L.lib.krill_prefix_set_disk(self.handle, _enc(cache_dir), budget_bytes))

    def wait_for_disk_writes(self):
        check(L.lib.krill_prefix_wait_disk(self.handle))

    @property
    def disk_count(self) -> int:
        v = C.c_int32()
        check(L.lib.krill_prefix_disk_count(self.handle, C.byref(v)))
        return v.value

    def close(self):
        if self.handle:
            check(L.lib.krill_prefix_destroy(self.handle))
            self.handle = None

    def store_quantized(self, tokens, model_id: str, seq: Sequence_, media_hash: Optional[str] = None):
        check(L.lib.krill_prefix_store(self.handle, seq.handle, _tok_array(tokens), len(tokens),
                                       _enc(model_id), _enc(media_hash)))

    def _lookup(self, fn, tokens, model_id, media_hash):
        e = C.c_void_p()
        n = C.c_int64()
        st = check(fn(self.handle, _tok_array(tokens), len(tokens), _enc(model_id), _enc(media_hash),
                      C.byref(e), C.byref(n)), allow=(L.KRILL_OK, L.KRILL_ERR_NOT_FOUND))
        if st == L.KRILL_ERR_NOT_FOUND:
            return None
        return QuantizedPrefixCacheHit(self, e, n.value)

    def lookup_quantized(self, tokens, model_id: str, media_hash: Optional[str] = None):
        return self._lookup(L.lib.krill_prefix_lookup, tokens, model_id, media_hash)

    def lookup_longest_prefix_quantized(self, tokens, model_id: str, media_hash: Optional[str] = None):
        return self._lookup(L.lib.krill_prefix_lookup_longest, tokens, model_id, media_hash)

    def clear(self):
        check(L.lib.krill_prefix_clear(self.handle))

    @property
    def memory_count(self) -> int:
        v = C.c_int32()
        check(L.lib.krill_prefix_memory_count(self.handle, C.byref(v)))
        return v.value

    def peer_fetch(self, src: "PrefixCache", hit: QuantizedPrefixCacheHit, stream=None):
        """Copy a hit owned by another GPU's cache into this one over NVLink."""
        e = C.c_void_p()
        check(L.lib.krill_prefix_peer_fetch(self.handle, src.handle, hit.entry, _stream(stream),
                                            C.byref(e)))
        return QuantizedPrefixCacheHit(self, e, hit.prefix_length)

    def describe(self, hit: QuantizedPrefixCacheHit) -> bytes:
        """Entry descriptor for krill_prefix_import in another process."""
        n = C.c_int64()
        check(L.lib.krill_prefix_entry_describe(self.handle, hit.entry, None, 0, C.byref(n)))
        buf = C.create_string_buffer(n.value)
        check(L.lib.krill_prefix_entry_describe(self.handle, hit.entry, buf, n.value, C.byref(n)))
        return buf.raw[: n.value]

    def import_entry(self, pool_handle: bytes, desc: bytes, stream=None) -> QuantizedPrefixCacheHit:
        """Copy an entry owned by another process's pool (IPC handle +
        descriptor) into this cache over NVLink; returns a held hit."""
        e = C.c_void_p()
        check(L.lib.krill_prefix_import(self.handle, pool_handle, desc, len(desc), _stream(stream),
                                        C.byref(e)))
        n = C.c_int64()
        check(L.lib.krill_prefix_entry_length(e, C.byref(n)))
        return QuantizedPrefixCacheHit(self, e, n.value)


def prefix_key(tokens, model_id: str, media_hash: Optional[str] = None, dtype_tag: int = 2) -> int:
    return L.lib.krill_prefix_key(_tok_array(tokens), len(tokens), _enc(model_id), _enc(media_hash),
                                  dtype_tag)
