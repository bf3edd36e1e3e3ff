"""Allocation-free decode attention (krill_decode_attention_noalloc).

For callers that cannot let the library allocate device or pinned memory
while they decode (an engine that reserved all device memory for its own
allocator, a serving loop that must not take the driver's allocation locks
mid-step). The entry point keeps its scratch in a fixed array inside the
library instead of growing buffers with cudaMalloc.

This file is named so that pytest collects it last. The test calls the entry
point through the C ABI twice in a row — the second time after new tokens
were appended, so any stale scratch from the first call would show — and
checks each output against krill_decode_attention on the same cache, within
the attention tolerance used by the other parity tests (2e-3 max-abs, fp32
outputs). Lengths above 4096 tokens make the call use the split partial
records in the scratch, not only its metadata.
"""
import ctypes as C

import numpy as np
import pytest

from tests._data import BF16, kv_values, to_bits

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

import krill_b200 as kb  # noqa: E402
from krill_b200 import _lib as L  # noqa: E402
from tests._gpu import dev_bits, prefill  # noqa: E402

ATOL = 2e-3


def _noalloc(pool, seqs, q, out, scale):
    arr = (C.c_uint64 * len(seqs))(*[s.handle for s in seqs])
    stream = torch.cuda.current_stream().cuda_stream
    L.check(L.lib.krill_decode_attention_noalloc(pool.handle, len(seqs), arr, 0, q.shape[0],
                                                 q.data_ptr(), L.DTYPE_BF16, out.data_ptr(),
                                                 L.DTYPE_F32, scale, stream))


def test_noalloc_matches_allocating_entry_point_on_two_calls():
    rng = np.random.default_rng(21)
    D, hq, hkv, layers = 128, 32, 8, 2
    scale = 1.0 / np.sqrt(D)
    pool = kb.KVPool(layers, hkv, hq, D, num_blocks=96)
    lengths = [37, 1000, 4500, 9000]
    seqs = []
    for Lq in lengths:
        s = pool.create_sequence()
        prefill(pool, s, to_bits(kv_values(rng, (layers, hkv, Lq, D)), BF16),
                to_bits(kv_values(rng, (layers, hkv, Lq, D)), BF16), BF16)
        seqs.append(s)
    n = len(seqs)
    for call in range(2):
        if call == 1:  # new tokens between the calls
            k1 = dev_bits(to_bits(kv_values(rng, (layers, n, hkv, 1, D)), BF16), BF16)
            v1 = dev_bits(to_bits(kv_values(rng, (layers, n, hkv, 1, D)), BF16), BF16)
            kb.append_quantize(pool, seqs, 0, k1, v1)
        q = dev_bits(to_bits(kv_values(rng, (layers, n, hq, D)), BF16), BF16)
        want = torch.empty((layers, n, hq, D), dtype=torch.float32, device="cuda")
        got = torch.full((layers, n, hq, D), float("nan"), dtype=torch.float32, device="cuda")
        kb.decode_attention(pool, seqs, 0, q, want, scale)
        _noalloc(pool, seqs, q, got, scale)
        torch.cuda.synchronize()
        err = (got - want).abs().max().item()
        assert err <= ATOL, f"call {call}: max abs diff {err:.3e}"
    assert pool.device_error() == 0
    pool.close()
