"""Allocation-free decode attention (krill_decode_attention_noalloc).

Some callers cannot let the library allocate while they decode: an engine
that reserved all device memory for its own allocator (a cudaMalloc from the
library would fail or fragment its arena), or a serving loop that must not
take the driver's allocation locks in the middle of a step. The entry point
keeps its scratch in a fixed array inside the library instead of growing
buffers with cudaMalloc.

This file is named so that pytest collects it last. Each parity test calls
the entry point through the C ABI twice in a row — the second time after new
tokens were appended, so stale scratch from the first call would show — and
checks each output against the float64 oracle (tolerance 2e-3 max-abs on
fp32 output, as in the other attention parity tests) and against
krill_decode_attention on the same cache. Lengths above 4096 tokens make the
call use the split partial records in the scratch, not only its metadata.
Further tests: the first call on a fresh pool, before any allocating call,
leaves the device's free memory unchanged; a call that needs more scratch
than the array holds is refused with KRILL_ERR_INVALID and the byte count,
without launching anything.
"""
import ctypes as C
import math
import re

import numpy as np
import pytest

import oracle
from tests._data import BF16, F16, kv_values, to_bits

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

import krill_b200 as kb  # noqa: E402
from krill_b200 import _lib as L  # noqa: E402
from tests._gpu import dev_bits, prefill  # noqa: E402

ATOL = 2e-3
SCRATCH = 16 * 1024 * 1024  # KRILL_NOALLOC_SCRATCH_BYTES


def _noalloc_rc(pool, seqs, q, q_dtype, out):
    arr = (C.c_uint64 * len(seqs))(*[s.handle for s in seqs])
    stream = torch.cuda.current_stream().cuda_stream
    scale = 1.0 / math.sqrt(pool.head_dim) if pool.head_dim != 256 else 1.0
    return L.lib.krill_decode_attention_noalloc(pool.handle, len(seqs), arr, 0, q.shape[0],
                                                q.data_ptr(), q_dtype, out.data_ptr(),
                                                L.DTYPE_F32, scale, stream), scale


def _noalloc(pool, seqs, q, q_dtype, out):
    rc, scale = _noalloc_rc(pool, seqs, q, q_dtype, out)
    L.check(rc)
    return scale


def _make(D, G, hq, hkv, layers, dtype, lengths, window=0, seed=21):
    rng = np.random.default_rng(seed)
    blocks = sum((Lq + 8) // 256 + 2 for Lq in lengths) + 16
    pool = kb.KVPool(layers, hkv, hq, D, num_blocks=blocks, group_size=G, window=window)
    seqs, kh, vh = [], [], []
    for Lq in lengths:
        s = pool.create_sequence()
        k = to_bits(kv_values(rng, (layers, hkv, Lq, D)), dtype)
        v = to_bits(kv_values(rng, (layers, hkv, Lq, D)), dtype)
        prefill(pool, s, k, v, dtype, chunk=256 if window else 0)
        seqs.append(s)
        kh.append(k)
        vh.append(v)
    return rng, pool, seqs, kh, vh


def _check_oracle(got, qb, kh, vh, dtype, G, scale, window):
    for i in range(len(kh)):
        for layer in range(got.shape[0]):
            kk, vv = kh[i][layer], vh[i][layer]
            if window:
                kk, vv = kk[:, -window:], vv[:, -window:]
            ck, sk, zk = oracle.quantize(kk, dtype, G)
            cv, sv, zv = oracle.quantize(vv, dtype, G)
            ref = oracle.reference_attention(ck, sk, zk, cv, sv, zv, qb[layer, i], dtype, G, scale)
            err = float(np.abs(got[layer, i] - ref).max())
            assert err <= ATOL, f"seq {i} (L={kk.shape[1]}) layer {layer}: max err {err:.3e}"


@pytest.mark.parametrize("D,G,hq,hkv,layers,dtype,lengths,window", [
    (128, 64, 32, 8, 2, BF16, [37, 1000, 4500, 9000], 0),   # Llama-3.1-8B shape, split pieces
    (64, 64, 32, 8, 16, F16, [2048], 0),                     # Llama-3.2-1B shape
    (256, 64, 8, 4, 2, F16, [300, 1500, 5000], 1024),        # sliding window 1024, ring wrapped
])
def test_noalloc_matches_oracle_on_two_calls(D, G, hq, hkv, layers, dtype, lengths, window):
    rng, pool, seqs, kh, vh = _make(D, G, hq, hkv, layers, dtype, lengths, window)
    n = len(seqs)
    for call in range(2):
        if call == 1:  # new tokens between the calls
            k1 = to_bits(kv_values(rng, (layers, n, hkv, 1, D)), dtype)
            v1 = to_bits(kv_values(rng, (layers, n, hkv, 1, D)), dtype)
            kb.append_quantize(pool, seqs, 0, dev_bits(k1, dtype), dev_bits(v1, dtype))
            for i in range(n):
                kh[i] = np.concatenate([kh[i], k1[:, i]], axis=2)
                vh[i] = np.concatenate([vh[i], v1[:, i]], axis=2)
        qb = to_bits(kv_values(rng, (layers, n, hq, D)), dtype)
        q = dev_bits(qb, dtype)
        got = torch.full((layers, n, hq, D), float("nan"), dtype=torch.float32, device="cuda")
        scale = _noalloc(pool, seqs, q, dtype, got)
        want = torch.empty_like(got)
        kb.decode_attention(pool, seqs, 0, q, want, scale)
        torch.cuda.synchronize()
        g = got.cpu().numpy().astype(np.float64)
        _check_oracle(g, qb, kh, vh, dtype, G, scale, window)
        diff = float(np.abs(g - want.cpu().numpy()).max())
        assert diff <= ATOL, f"call {call}: differs from krill_decode_attention by {diff:.3e}"
    assert pool.device_error() == 0
    pool.close()


def test_noalloc_first_calls_allocate_nothing():
    """On a fresh pool the no-alloc call comes before any allocating call and
    the device's free memory is the same after two calls as before them. A
    throwaway pool of the same shape runs the same kernels first, so that
    loading their code (lazy module loading) is not counted."""
    D, G, hq, hkv, layers = 128, 64, 32, 8, 2
    lengths = [700, 5000]
    _, warm, wseqs, _, _ = _make(D, G, hq, hkv, layers, BF16, lengths, seed=3)
    rng, pool, seqs, kh, vh = _make(D, G, hq, hkv, layers, BF16, lengths, seed=4)
    n = len(seqs)
    qb = to_bits(kv_values(rng, (layers, n, hq, D)), BF16)
    q = dev_bits(qb, BF16)
    outs = [torch.full((layers, n, hq, D), float("nan"), dtype=torch.float32, device="cuda")
            for _ in range(2)]
    _noalloc(warm, wseqs, q, BF16, outs[0])
    torch.cuda.synchronize()
    warm.close()
    free0 = torch.cuda.mem_get_info()[0]
    for out in outs:
        scale = _noalloc(pool, seqs, q, BF16, out)
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info()[0]
    assert free1 == free0, f"free device memory changed by {free0 - free1} bytes"
    for out in outs:
        _check_oracle(out.cpu().numpy().astype(np.float64), qb, kh, vh, BF16, G, scale, 0)
    pool.close()


def test_noalloc_rejects_oversized_call_without_launching():
    """32 layers x 8 sequences of 8,193 tokens split into 3 pieces each: the
    partial records need more than the 16 MiB scratch, so the call returns
    KRILL_ERR_INVALID with the byte count and launches no kernel."""
    D, hq, hkv, layers, Lq, n = 128, 32, 8, 32, 8193, 8
    pool = kb.KVPool(layers, hkv, hq, D, num_blocks=n * 33 + 4)
    kv = torch.zeros((layers, 1, hkv, Lq, D), dtype=torch.bfloat16, device="cuda")
    seqs = [pool.create_sequence() for _ in range(n)]
    for s in seqs:
        kb.append_quantize(pool, [s], 0, kv, kv)
    del kv
    q = torch.zeros((layers, n, hq, D), dtype=torch.bfloat16, device="cuda")
    out = torch.full((layers, n, hq, D), float("nan"), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    pool.kernel_count()
    rc, _ = _noalloc_rc(pool, seqs, q, BF16, out)
    assert rc == L.KRILL_ERR_INVALID
    msg = L.lib.krill_last_error_string().decode()
    m = re.search(r"needs (\d+) bytes of scratch", msg)
    assert m and int(m.group(1)) > SCRATCH, msg
    assert pool.kernel_count() == 0
    torch.cuda.synchronize()
    assert torch.isnan(out).all().item()
    pool.close()


def test_noalloc_refuses_a_stream_under_capture():
    """The metadata is copied from a host buffer that the next call
    overwrites, so a call on a stream being captured is refused (and
    enqueues nothing); the same call outside the capture then succeeds."""
    rng, pool, seqs, kh, vh = _make(128, 64, 32, 8, 1, BF16, [300], seed=9)
    qb = to_bits(kv_values(rng, (1, 1, 32, 128)), BF16)
    q = dev_bits(qb, BF16)
    out = torch.full((1, 1, 32, 128), float("nan"), dtype=torch.float32, device="cuda")
    side = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    torch.cuda.synchronize()
    with torch.cuda.stream(side):
        graph.capture_begin()
        try:
            rc, _ = _noalloc_rc(pool, seqs, q, BF16, out)
            out.add_(0.0)  # keeps the captured graph non-empty
        finally:
            graph.capture_end()
    assert rc == L.KRILL_ERR_INVALID
    assert "capture" in L.lib.krill_last_error_string().decode()
    del graph
    scale = _noalloc(pool, seqs, q, BF16, out)
    torch.cuda.synchronize()
    _check_oracle(out.cpu().numpy().astype(np.float64), qb, kh, vh, BF16, 64, scale, 0)
    pool.close()
