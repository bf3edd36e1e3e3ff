"""Fused quantize+append parity: codes, scales and zeros bit-exact with the
oracle restatement of QuantizedKVCache.quantizePerHead
(QuantizedKVCache.swift:181-197); dequantized snapshots bit-exact with
QuantizedKVCache.dequantize (:200-204)."""
import numpy as np
import pytest

import oracle
from tests._data import BF16, F16, kv_values, to_bits

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

import krill_b200 as kb  # noqa: E402
from tests._gpu import dev_bits, host_bits, prefill  # noqa: E402

CASES = [
    # D, G, dtype, variant, outliers
    (64, 64, F16, 0, False),
    (128, 64, BF16, 0, False),
    (128, 64, F16, 0, True),
    (128, 128, F16, 0, False),
    (256, 64, F16, 0, False),
    (256, 64, BF16, 0, True),
    (256, 256, BF16, 0, False),
    (128, 64, F16, 1, False),
    (128, 64, BF16, 1, True),
]


@pytest.mark.parametrize("D,G,dtype,variant,outliers", CASES)
def test_append_codes_bit_exact(D, G, dtype, variant, outliers):
    rng = np.random.default_rng(1000 + D + G + dtype * 7 + variant * 13)
    layers, hkv, hq = 2, 4, 8
    pool = kb.KVPool(layers, hkv, hq, D, num_blocks=32, group_size=G, quant_variant=variant)
    lengths = [1, 63, 64, 65, 300]
    seqs, kbits, vbits = [], [], []
    for L in lengths:
        s = pool.create_sequence()
        k = to_bits(kv_values(rng, (layers, hkv, L, D), outliers), dtype)
        v = to_bits(kv_values(rng, (layers, hkv, L, D), outliers), dtype)
        prefill(pool, s, k, v, dtype, chunk=97)
        seqs.append(s)
        kbits.append(k)
        vbits.append(v)
    # three batched single-token decode appends over all sequences
    for _ in range(3):
        k1 = to_bits(kv_values(rng, (layers, len(seqs), hkv, 1, D), outliers), dtype)
        v1 = to_bits(kv_values(rng, (layers, len(seqs), hkv, 1, D), outliers), dtype)
        kb.append_quantize(pool, seqs, 0, dev_bits(k1, dtype), dev_bits(v1, dtype))
        for i in range(len(seqs)):
            kbits[i] = np.concatenate([kbits[i], k1[:, i]], axis=2)
            vbits[i] = np.concatenate([vbits[i], v1[:, i]], axis=2)
    torch.cuda.synchronize()
    for i, s in enumerate(seqs):
        assert s.length(0) == lengths[i] + 3
        for layer in range(layers):
            snap = s.quantized_snapshot(layer)
            ck, sk, zk = oracle.quantize(kbits[i][layer], dtype, G, variant)
            cv, sv, zv = oracle.quantize(vbits[i][layer], dtype, G, variant)
            np.testing.assert_array_equal(snap.keys.cpu().numpy(), ck)
            np.testing.assert_array_equal(snap.values.cpu().numpy(), cv)
            np.testing.assert_array_equal(host_bits(snap.key_scales), sk)
            np.testing.assert_array_equal(host_bits(snap.key_zeros), zk)
            np.testing.assert_array_equal(host_bits(snap.value_scales), sv)
            np.testing.assert_array_equal(host_bits(snap.value_zeros), zv)
            kd, vd = s.snapshot(layer)
            np.testing.assert_array_equal(host_bits(kd), oracle.dequantize(ck, sk, zk, G))
            np.testing.assert_array_equal(host_bits(vd), oracle.dequantize(cv, sv, zv, G))
    pool.close()


def test_weyl_round_trip_bounds():
    """QuantizedKVCacheUnitTests (QuantizedKVCacheUnitTests.swift:38-84): the
    deterministic Weyl tensor round-trips within 1.5 steps + 1e-3 (positive)
    and + 1e-2 (mixed sign), through the GPU quantizer and dequantizer."""
    pool = kb.KVPool(1, 4, 4, 64, num_blocks=4, group_size=64)
    for lo, hi, slack in [(0.0, 10.0, 1e-3), (0.0, 5.0, 1e-3), (-64.0, 64.0, 1e-2), (-32.0, 64.0, 1e-2)]:
        total = 4 * 8 * 64
        span = max(hi - lo, 1e-3)
        i = np.arange(total, dtype=np.float32)
        frac = i * np.float32(0.6180339887) - np.floor(i * np.float32(0.6180339887))
        x = (np.float32(lo) + frac * np.float32(span)).reshape(1, 4, 8, 64)
        bits = to_bits(x, F16)
        s = pool.create_sequence()
        kb.append_quantize(pool, [s], 0, dev_bits(bits[:, None], F16), dev_bits(bits[:, None], F16))
        kd, _ = s.snapshot(0)
        ref = bits.view(np.float16).astype(np.float32)[0]
        err = np.abs(kd.float().cpu().numpy() - ref).max()
        assert err < (hi - lo) / 255.0 * 1.5 + slack, err
        s.release()
    pool.close()
