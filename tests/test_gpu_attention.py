"""Decode-attention parity: the fused int8 kernel vs the reference math
(full-cache fp16 dequantize, QuantizedKVCache.swift:71-74 + :200-204, then
SDPA with GQA, Gemma4Model.swift:516 / Attention.swift:95) evaluated in
float64 by the oracle.

Tolerance (written here, per the hot-path contract): max-abs 2e-3 on fp32
outputs; for f16/bf16 outputs 2e-3 plus one half-ulp of the output dtype at
the reference value (the rounding of the stored result itself).
"""
import math

import numpy as np
import pytest

import oracle
from tests._data import BF16, F16, kv_values, to_bits

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

import krill_b200 as kb  # noqa: E402
from tests._gpu import dev_bits, prefill  # noqa: E402

ATOL = 2e-3


def half_ulp(ref: np.ndarray, out_dtype) -> np.ndarray:
    if out_dtype == torch.float32:
        return np.zeros_like(ref)
    mant = 10 if out_dtype == torch.float16 else 7
    e = np.floor(np.log2(np.maximum(np.abs(ref), 2.0 ** -14)))
    return 0.5 * 2.0 ** (e - mant)


def run_case(D, G, hq, hkv, dtype, lengths, scale, out_dtype=torch.float32, window=0, split=256,
             outliers=False, layers=2, seed=0, impl=kb.ATTN_TENSOR_CORE, steps=2):
    rng = np.random.default_rng(seed)
    blocks = max(64, sum((L + steps) // 256 + 2 for L in lengths) + 8)
    pool = kb.KVPool(layers, hkv, hq, D, num_blocks=blocks, group_size=G, window=window,
                     split_tokens=split, attn_impl=impl)
    seqs, kb_all, vb_all = [], [], []
    for L in lengths:
        s = pool.create_sequence()
        k = to_bits(kv_values(rng, (layers, hkv, L, D), outliers), dtype)
        v = to_bits(kv_values(rng, (layers, hkv, L, D), outliers), dtype)
        if window:  # a windowed pool takes at most max_append tokens per call
            prefill(pool, s, k, v, dtype, chunk=256)
        else:
            prefill(pool, s, k, v, dtype)
        seqs.append(s)
        kb_all.append(k)
        vb_all.append(v)
    n = len(seqs)
    worst = 0.0
    for _ in range(steps):
        k1 = to_bits(kv_values(rng, (layers, n, hkv, 1, D), outliers), dtype)
        v1 = to_bits(kv_values(rng, (layers, n, hkv, 1, D), outliers), dtype)
        qb = to_bits(kv_values(rng, (layers, n, hq, D)), dtype)
        out = torch.empty((layers, n, hq, D), dtype=out_dtype, device="cuda")
        kb.decode_step(pool, seqs, 0, dev_bits(k1, dtype), dev_bits(v1, dtype), dev_bits(qb, dtype),
                       out, scale)
        torch.cuda.synchronize()
        got = out.float().cpu().numpy().astype(np.float64)
        for i in range(n):
            kb_all[i] = np.concatenate([kb_all[i], k1[:, i]], axis=2)
            vb_all[i] = np.concatenate([vb_all[i], v1[:, i]], axis=2)
            for layer in range(layers):
                kk = kb_all[i][layer]
                vv = vb_all[i][layer]
                if window:
                    kk = kk[:, -window:]
                    vv = vv[:, -window:]
                ck, sk, zk = oracle.quantize(kk, dtype, G)
                cv, sv, zv = oracle.quantize(vv, dtype, G)
                ref = oracle.reference_attention(ck, sk, zk, cv, sv, zv, qb[layer, i], dtype, G, scale)
                err = np.abs(got[layer, i] - ref)
                tol = ATOL + half_ulp(ref, out_dtype)
                assert np.all(err <= tol), (
                    f"seq {i} (L={kk.shape[1]}) layer {layer}: max err {err.max():.3e}")
                worst = max(worst, float(err.max()))
    pool.close()
    return worst


@pytest.mark.parametrize("D,G,hq,hkv,dtype,scale", [
    (64, 64, 32, 8, F16, 1 / 8),          # Llama-3.2-1B shape (config 1)
    (128, 64, 32, 8, BF16, 1 / math.sqrt(128)),  # Llama-3.1-8B shape (config 2)
    (128, 64, 32, 4, BF16, 1 / math.sqrt(128)),  # Qwen3-30B-A3B KV shape (GQA 8, config 4)
    (256, 64, 8, 4, F16, 1.0),            # Gemma-style D=256, GQA 2, scale 1 (config 5)
    (128, 128, 16, 16, F16, 1 / math.sqrt(128)),  # G = D (strict reference scheme), MHA, 2 rounds
    (128, 64, 8, 2, BF16, 1 / math.sqrt(128)),   # 2 kv heads: 4 warps merge per head
    (64, 64, 8, 1, F16, 1 / 8),                  # MQA: 8 warps merge on one head
    (256, 256, 16, 2, BF16, 1.0),                # D=256, G=D, 2 kv heads
])
def test_attention_ragged(D, G, hq, hkv, dtype, scale):
    run_case(D, G, hq, hkv, dtype, [1, 5, 63, 64, 65, 200, 700], scale)


def test_attention_long_split():
    # several split-K items per unit, combined by the last CTA
    run_case(128, 64, 32, 8, BF16, [3000, 1100], 1 / math.sqrt(128), split=512, layers=1)


@pytest.mark.parametrize("D,G,hq,hkv,dtype,lengths,layers", [
    (128, 64, 32, 8, BF16, [20000], 1),   # one long sequence: pieces merged by the last arriver
    (64, 64, 32, 8, F16, [2048], 16),     # configs[0] shape: one kv head per item, whole sequence
    (256, 64, 8, 4, F16, [9000, 70], 2),  # D = 256, GQA 2, ragged
    (128, 128, 16, 16, F16, [5000], 1),   # MHA: several head rounds per item
    (64, 64, 8, 1, F16, [12000], 1),      # MQA: 8 warps share the one head
])
def test_attention_latency_bound_adaptive(D, G, hq, hkv, dtype, lengths, layers):
    """Adaptive splitting on small batches: the planner's latency-bound regime
    (head-split items, pieces merged in the decode kernel by the piece that
    arrives last, one item per CTA)."""
    scale = 1 / math.sqrt(D)
    run_case(D, G, hq, hkv, dtype, lengths, scale, split=0, layers=layers, steps=2)


def test_attention_outliers_gqa8():
    run_case(128, 64, 32, 4, BF16, [900, 33], 1 / math.sqrt(128), outliers=True, layers=1)


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.bfloat16])
def test_attention_low_precision_out(out_dtype):
    run_case(128, 64, 32, 8, BF16, [17, 300], 1 / math.sqrt(128), out_dtype=out_dtype, layers=1)


def test_attention_windowed():
    # RotatingKVCache semantics: attend the last `window` positions only
    run_case(256, 64, 8, 4, F16, [10, 100, 300, 700], 1.0, window=128, layers=2, steps=3)


def test_batch_invariance_bit_exact():
    """BatchedDecodeLiveTests.swift:533-576: a row's output does not depend
    on the other rows (R=1 batched == solo, cross-row isolation), bit for bit."""
    rng = np.random.default_rng(5)
    D, hq, hkv, layers = 128, 32, 8, 2
    pool = kb.KVPool(layers, hkv, hq, D, num_blocks=64, split_tokens=256)
    lengths = [40, 900, 2000]
    seqs = []
    for L in lengths:
        s = pool.create_sequence()
        prefill(pool, s, to_bits(kv_values(rng, (layers, hkv, L, D)), BF16),
                to_bits(kv_values(rng, (layers, hkv, L, D)), BF16), BF16)
        seqs.append(s)
    qb = to_bits(kv_values(rng, (layers, 3, hq, D)), BF16)
    q = dev_bits(qb, BF16)
    out_all = torch.empty((layers, 3, hq, D), dtype=torch.float32, device="cuda")
    kb.decode_attention(pool, seqs, 0, q, out_all, 0.1)
    for i in range(3):
        out_one = torch.empty((layers, 1, hq, D), dtype=torch.float32, device="cuda")
        kb.decode_attention(pool, [seqs[i]], 0, q[:, i:i + 1].contiguous(), out_one, 0.1)
        torch.cuda.synchronize()
        assert torch.equal(out_one[:, 0], out_all[:, i])
    pool.close()


def test_neighbor_content_isolation_bit_exact():
    """BatchedDecodeLiveTests.swift:533-546 (cross-row isolation at a fixed
    batch width): with the adaptive decomposition, a row's output is
    bit-identical when only its neighbors' K/V/q contents change."""
    D, hq, hkv, layers = 128, 32, 8, 2
    lengths = [700, 1500, 333]
    outs = []
    for neighbor_seed in (11, 12):
        rng_row = np.random.default_rng(3)
        rng_nb = np.random.default_rng(neighbor_seed)
        pool = kb.KVPool(layers, hkv, hq, D, num_blocks=64)  # adaptive split
        seqs = []
        for i, L in enumerate(lengths):
            rng = rng_row if i == 0 else rng_nb
            s = pool.create_sequence()
            prefill(pool, s, to_bits(kv_values(rng, (layers, hkv, L, D)), BF16),
                    to_bits(kv_values(rng, (layers, hkv, L, D)), BF16), BF16)
            seqs.append(s)
        qrow = to_bits(kv_values(np.random.default_rng(4), (layers, 1, hq, D)), BF16)
        qnb = to_bits(kv_values(rng_nb, (layers, 2, hq, D)), BF16)
        q = dev_bits(np.ascontiguousarray(np.concatenate([qrow, qnb], axis=1)), BF16)
        out = torch.empty((layers, 3, hq, D), dtype=torch.float32, device="cuda")
        kb.decode_attention(pool, seqs, 0, q, out, 0.1)
        torch.cuda.synchronize()
        outs.append(out[:, 0].clone())
        pool.close()
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("D,G,hq,hkv,dtype,scale", [
    (64, 64, 32, 8, F16, 1 / 8),
    (128, 64, 32, 8, BF16, 1 / math.sqrt(128)),
    (128, 64, 32, 4, BF16, 1 / math.sqrt(128)),
    (256, 64, 8, 4, F16, 1.0),
    (64, 64, 8, 8, F16, 1 / 8),
])
def test_attention_cuda_core_variant(D, G, hq, hkv, dtype, scale):
    """The CUDA-core variant (attn_impl = CUDA_CORE) meets the same tolerance."""
    run_case(D, G, hq, hkv, dtype, [1, 63, 65, 300, 1100], scale, impl=kb.ATTN_CUDA_CORE, split=512)


def test_attention_cuda_core_windowed():
    run_case(256, 64, 8, 4, F16, [10, 300, 700], 1.0, window=128, impl=kb.ATTN_CUDA_CORE, steps=2)


@pytest.mark.parametrize("dtype", [F16, BF16])
def test_attention_large_scales(dtype):
    """Groups whose range exceeds 64 * 255 store scales >= 64, where the
    one-fma dequantization would overflow: the pool's large-scale flag must
    route the launch to the exact two-rounding path. K stays N(0, 1); a tenth
    of the tokens carry V of magnitude up to 12000. Tolerance relative to the
    output magnitude (f16 P weights on values of that size)."""
    rng = np.random.default_rng(7)
    D, G, hq, hkv, layers = 128, 64, 32, 8, 1
    scale = 1 / math.sqrt(D)
    pool = kb.KVPool(layers, hkv, hq, D, num_blocks=16, group_size=G)
    lengths = [300, 77]
    seqs, K, V = [], [], []
    for L in lengths:
        s = pool.create_sequence()
        k = to_bits(kv_values(rng, (layers, hkv, L, D)), dtype)
        vf = rng.standard_normal((layers, hkv, L, D))
        big = rng.random(L) < 0.1
        vf[:, :, big, :] = rng.uniform(-12000, 12000, size=vf[:, :, big, :].shape)
        v = to_bits(vf, dtype)
        prefill(pool, s, k, v, dtype)
        seqs.append(s)
        K.append(k)
        V.append(v)
    _, sv, _ = oracle.quantize(V[0][0], dtype, G)
    assert (oracle.bits_to_f64(sv, F16) >= 64).any()  # the case under test
    n = len(seqs)
    qb = to_bits(kv_values(rng, (layers, n, hq, D)), dtype)
    out = torch.empty((layers, n, hq, D), dtype=torch.float32, device="cuda")
    kb.decode_attention(pool, seqs, 0, dev_bits(qb, dtype), out, scale)
    torch.cuda.synchronize()
    assert pool.device_error() == 0
    got = out.cpu().numpy().astype(np.float64)
    for i in range(n):
        ck, sk, zk = oracle.quantize(K[i][0], dtype, G)
        cv, sv, zv = oracle.quantize(V[i][0], dtype, G)
        ref = oracle.reference_attention(ck, sk, zk, cv, sv, zv, qb[0, i], dtype, G, scale)
        err = np.abs(got[0, i] - ref).max()
        assert np.isfinite(got[0, i]).all()
        assert err <= ATOL * max(1.0, np.abs(ref).max()), f"seq {i}: max err {err:.3e}"
    pool.close()
