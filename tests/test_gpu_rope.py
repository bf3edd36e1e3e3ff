"""Fused RoPE + quantize + append: the new K is rotated at each token's
position (MLXFast.RoPE with traditional: false, applied before
cache.update, Gemma4Model.swift:502-509; per-row positions as in
Attention.swift:13-20), rounded to the input dtype and quantized. Codes,
scales and zeros must equal the oracle's (rotate in float32, round, quantize)
bit for bit; V is appended unrotated."""
import numpy as np
import pytest

import oracle
from tests._data import BF16, F16, kv_values, to_bits

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

import krill_b200 as kb  # noqa: E402
from tests._gpu import dev_bits, host_bits  # noqa: E402


@pytest.mark.parametrize("D,G,dtype,base", [
    (128, 64, BF16, 500000.0),   # Llama-3.1 rope_theta
    (64, 64, F16, 10000.0),
    (256, 64, F16, 1000000.0),
    (128, 128, F16, 10000.0),
])
def test_rope_append_matches_oracle(D, G, dtype, base):
    rng = np.random.default_rng(5)
    layers, hkv, hq = 2, 4, 8
    rows = 1024
    cos, sin = oracle.rope_table(base, D, rows)
    dcos, dsin = torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()
    pool = kb.KVPool(layers, hkv, hq, D, num_blocks=32, group_size=G)
    starts = [0, 37, 300]
    seqs, K, V = [], [], []
    for L in starts:
        s = pool.create_sequence()
        if L:  # prefill through the RoPE path: the cache holds rotated K
            k0 = to_bits(kv_values(rng, (layers, hkv, L, D)), dtype)
            v0 = to_bits(kv_values(rng, (layers, hkv, L, D)), dtype)
            kb.append_quantize(pool, [s], 0, dev_bits(k0[:, None], dtype), dev_bits(v0[:, None], dtype),
                               rope=(dcos, dsin))
            K.append(np.stack([oracle.apply_rope(k0[l], dtype, cos, sin, np.arange(L))
                               for l in range(layers)]))
            V.append(v0)
        else:
            K.append(np.zeros((layers, hkv, 0, D), np.uint16))
            V.append(np.zeros((layers, hkv, 0, D), np.uint16))
        seqs.append(s)
    for n_new in (1, 20):
        k1 = to_bits(kv_values(rng, (layers, len(seqs), hkv, n_new, D)), dtype)
        v1 = to_bits(kv_values(rng, (layers, len(seqs), hkv, n_new, D)), dtype)
        kb.append_quantize(pool, seqs, 0, dev_bits(k1, dtype), dev_bits(v1, dtype), rope=(dcos, dsin))
        torch.cuda.synchronize()
        for i, s in enumerate(seqs):
            L0 = K[i].shape[2]
            pos = np.arange(L0, L0 + n_new)
            K[i] = np.concatenate([K[i], np.stack([oracle.apply_rope(k1[l, i], dtype, cos, sin, pos)
                                                    for l in range(layers)])], axis=2)
            V[i] = np.concatenate([V[i], v1[:, i]], axis=2)
    for i, s in enumerate(seqs):
        for layer in range(layers):
            snap = s.quantized_snapshot(layer)
            ck, sk, zk = oracle.quantize(K[i][layer], dtype, G)
            cv, sv, zv = oracle.quantize(V[i][layer], dtype, G)
            np.testing.assert_array_equal(snap.keys.cpu().numpy(), ck)
            np.testing.assert_array_equal(host_bits(snap.key_scales), sk)
            np.testing.assert_array_equal(host_bits(snap.key_zeros), zk)
            np.testing.assert_array_equal(snap.values.cpu().numpy(), cv)
            np.testing.assert_array_equal(host_bits(snap.value_scales), sv)
    pool.close()


def test_rope_position_beyond_table_is_rejected():
    pool = kb.KVPool(1, 4, 8, 128, num_blocks=8)
    cos, sin = oracle.rope_table(10000.0, 128, 16)
    dcos, dsin = torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()
    s = pool.create_sequence()
    k = torch.zeros((1, 1, 4, 17, 128), dtype=torch.float16, device="cuda")
    with pytest.raises(kb.KrillError):
        kb.append_quantize(pool, [s], 0, k, k, rope=(dcos, dsin))
    assert s.length(0) == 0
    pool.close()
