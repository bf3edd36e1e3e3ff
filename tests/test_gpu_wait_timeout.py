"""Bounded device waits: a wait that runs out ends the launch with an error
status instead of hanging the GPU.

The pool is created with a 1 ms wait limit and its test switch
(krill_pool_test_stall) makes an otherwise idle warp of CTA 0 wait for a
shared-memory word that nothing sets: the wait runs out after the limit,
raises KRILL_DEVICE_ERR_TIMEOUT in the pool's device error flag, and the
launch ends. Nothing faults or traps. The test checks that
the launch ends well within a second, that the flag reports the timeout (and
is cleared by reading it), and that the context stays usable: the same pool
and a fresh one then give results within the attention tolerance of the
oracle.
"""
import math
import time

import numpy as np
import pytest

import oracle
from tests._data import BF16, kv_values, to_bits

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

import krill_b200 as kb  # noqa: E402
from krill_b200 import _lib as L  # noqa: E402
from tests._gpu import dev_bits, prefill  # noqa: E402

ATOL = 2e-3
D, G, HQ, HKV, LAYERS = 128, 64, 32, 8, 2


def _pool_with(lengths, seed, **kw):
    rng = np.random.default_rng(seed)
    pool = kb.KVPool(LAYERS, HKV, HQ, D, num_blocks=64, group_size=G, **kw)
    seqs, data = [], []
    for Lq in lengths:
        s = pool.create_sequence()
        k = to_bits(kv_values(rng, (LAYERS, HKV, Lq, D)), BF16)
        v = to_bits(kv_values(rng, (LAYERS, HKV, Lq, D)), BF16)
        prefill(pool, s, k, v, BF16)
        seqs.append(s)
        data.append((k, v))
    qb = to_bits(kv_values(rng, (LAYERS, len(seqs), HQ, D)), BF16)
    return pool, seqs, data, qb


def _check(out, data, qb, scale):
    got = out.cpu().numpy().astype(np.float64)
    for i, (k, v) in enumerate(data):
        for layer in range(LAYERS):
            ck, sk, zk = oracle.quantize(k[layer], BF16, G)
            cv, sv, zv = oracle.quantize(v[layer], BF16, G)
            ref = oracle.reference_attention(ck, sk, zk, cv, sv, zv, qb[layer, i], BF16, G, scale)
            err = float(np.abs(got[layer, i] - ref).max())
            assert err <= ATOL, f"seq {i} layer {layer}: max err {err:.3e}"


def test_wait_runs_out_with_error_status_and_context_stays_usable():
    scale = 1 / math.sqrt(D)
    pool, seqs, data, qb = _pool_with([700, 3000], seed=41, wait_timeout_us=1000)
    q = dev_bits(qb, BF16)
    out = torch.empty((LAYERS, len(seqs), HQ, D), dtype=torch.float32, device="cuda")
    kb.decode_attention(pool, seqs, 0, q, out, scale)  # loads the kernel
    torch.cuda.synchronize()
    assert pool.device_error() == 0

    pool.test_stall(True)
    t0 = time.perf_counter()
    kb.decode_attention(pool, seqs, 0, q, out, scale)
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    pool.test_stall(False)
    flag = pool.device_error()
    assert flag & L.DEVICE_ERR_TIMEOUT, f"device error flag {flag}"
    assert pool.device_error() == 0, "reading the flag clears it"
    assert elapsed < 0.5, f"the stalled launch took {elapsed:.3f} s with a 1 ms wait limit"

    # the same pool, the switch off: correct again
    out.fill_(float("nan"))
    kb.decode_attention(pool, seqs, 0, q, out, scale)
    torch.cuda.synchronize()
    assert pool.device_error() == 0
    _check(out, data, qb, scale)
    pool.close()

    # a fresh pool with the default limit
    pool2, seqs2, data2, qb2 = _pool_with([1500], seed=42)
    out2 = torch.empty((LAYERS, 1, HQ, D), dtype=torch.float32, device="cuda")
    kb.decode_attention(pool2, seqs2, 0, dev_bits(qb2, BF16), out2, scale)
    torch.cuda.synchronize()
    assert pool2.device_error() == 0
    _check(out2, data2, qb2, scale)
    pool2.close()

