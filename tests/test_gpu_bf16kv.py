"""The raw bf16 pool format (the unquantized KVCache of
Sources/KrillCache/KVCache.swift:94, kept to compare against the int8 path):
bf16 K/V appended unchanged, decode attention on bf16 tensor cores for q·Kᵀ
and f16 for ·V. Reference: float64 SDPA with GQA over the same bf16 K/V.
Tolerance: max-abs 2e-3 on fp32 outputs (plus one half-ulp of the output
dtype for f16/bf16 outputs)."""
import math

import numpy as np
import pytest

import oracle
from tests._data import BF16, kv_values, to_bits

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

import krill_b200 as kb  # noqa: E402
from tests._gpu import dev_bits, prefill  # noqa: E402
from tests.test_gpu_attention import ATOL, half_ulp  # noqa: E402


def run_bf16(D, hq, hkv, lengths, scale, window=0, layers=2, split=0, out_dtype=torch.float32,
             steps=2, seed=0):
    rng = np.random.default_rng(seed)
    pool = kb.KVPool(layers, hkv, hq, D, num_blocks=80, window=window, split_tokens=split,
                     kv_format=kb.KV_BF16)
    seqs, K, V = [], [], []
    for L in lengths:
        s = pool.create_sequence()
        k = to_bits(kv_values(rng, (layers, hkv, L, D)), BF16)
        v = to_bits(kv_values(rng, (layers, hkv, L, D)), BF16)
        prefill(pool, s, k, v, BF16, chunk=256 if window else 0)
        seqs.append(s)
        K.append(k)
        V.append(v)
    n = len(seqs)
    for _ in range(steps):
        k1 = to_bits(kv_values(rng, (layers, n, hkv, 1, D)), BF16)
        v1 = to_bits(kv_values(rng, (layers, n, hkv, 1, D)), BF16)
        qb = to_bits(kv_values(rng, (layers, n, hq, D)), BF16)
        out = torch.empty((layers, n, hq, D), dtype=out_dtype, device="cuda")
        kb.decode_step(pool, seqs, 0, dev_bits(k1, BF16), dev_bits(v1, BF16), dev_bits(qb, BF16),
                       out, scale)
        torch.cuda.synchronize()
        assert pool.device_error() == 0
        got = out.float().cpu().numpy().astype(np.float64)
        for i in range(n):
            K[i] = np.concatenate([K[i], k1[:, i]], axis=2)
            V[i] = np.concatenate([V[i], v1[:, i]], axis=2)
            for layer in range(layers):
                kk, vv = K[i][layer], V[i][layer]
                if window:
                    kk, vv = kk[:, -window:], vv[:, -window:]
                ref = oracle.sdpa_f64(oracle.bf16_bits_to_f64(qb[layer, i]),
                                      oracle.bf16_bits_to_f64(kk), oracle.bf16_bits_to_f64(vv), scale)
                err = np.abs(got[layer, i] - ref)
                assert np.all(err <= ATOL + half_ulp(ref, out_dtype)), (
                    f"seq {i} L={kk.shape[1]} layer {layer}: max err {err.max():.3e}")
    pool.close()


@pytest.mark.parametrize("D,hq,hkv,scale", [
    (128, 32, 8, 1 / math.sqrt(128)),   # Llama-3.1-8B shape (configs[1] comparison)
    (128, 32, 4, 1 / math.sqrt(128)),   # GQA 8
    (64, 32, 8, 1 / 8),                 # D = 64
    (128, 8, 2, 1 / math.sqrt(128)),    # 2 kv heads: warps merge per head
])
def test_bf16kv_ragged(D, hq, hkv, scale):
    run_bf16(D, hq, hkv, [1, 5, 31, 32, 33, 200, 700], scale)


def test_bf16kv_long_split_and_windowed():
    run_bf16(128, 32, 8, [3000, 1100], 1 / math.sqrt(128), split=512, layers=1)
    run_bf16(128, 32, 8, [1500, 40], 1 / math.sqrt(128), window=1024, layers=1)


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.bfloat16])
def test_bf16kv_low_precision_out(out_dtype):
    run_bf16(128, 32, 8, [77, 300], 1 / math.sqrt(128), out_dtype=out_dtype, layers=1, steps=1)


def test_bf16kv_rejects_quantized_snapshot():
    pool = kb.KVPool(1, 8, 32, 128, num_blocks=4, kv_format=kb.KV_BF16)
    s = pool.create_sequence()
    k = to_bits(kv_values(np.random.default_rng(0), (1, 8, 10, 128)), BF16)
    prefill(pool, s, k, k, BF16)
    with pytest.raises(kb.KrillError):
        s.quantized_snapshot(0)
    pool.close()
