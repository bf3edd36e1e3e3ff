"""Multi-query verify attention over the int8 cache (speculative decoding;
the batched verify forward with buildBatchedVerifyMask,
BatchedDecode.swift:299-312): after n_query draft tokens are appended, query
j must equal single-token decode attention over the cache up to and
including draft j (oracle: the reference's dequantize + SDPA). Tolerance as
for decode attention: max-abs 2e-3 on fp32 outputs."""
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
from tests.test_gpu_attention import ATOL  # noqa: E402


@pytest.mark.parametrize("D,G,hq,hkv,dtype,nq", [
    (128, 64, 32, 8, BF16, 4),
    (128, 64, 32, 4, BF16, 2),
    (64, 64, 32, 8, F16, 5),
    (256, 64, 8, 4, F16, 3),
    (64, 64, 32, 8, F16, 3),   # 12 columns: two query tiles, the second half full
    (128, 64, 64, 8, BF16, 2), # GQA 8 with 8 kv heads: one query per tile, two tiles
])
def test_verify_matches_sequential_oracle(D, G, hq, hkv, dtype, nq):
    rng = np.random.default_rng(9)
    layers = 2
    scale = 1 / math.sqrt(D)
    pool = kb.KVPool(layers, hkv, hq, D, num_blocks=48, group_size=G)
    lengths = [1, 63, 64, 300, 700]
    seqs, K, V = [], [], []
    for L in lengths:
        s = pool.create_sequence()
        k = to_bits(kv_values(rng, (layers, hkv, L, D)), dtype)
        v = to_bits(kv_values(rng, (layers, hkv, L, D)), dtype)
        prefill(pool, s, k, v, dtype)
        seqs.append(s)
        K.append(k)
        V.append(v)
    n = len(seqs)
    kd = to_bits(kv_values(rng, (layers, n, hkv, nq, D)), dtype)
    vd = to_bits(kv_values(rng, (layers, n, hkv, nq, D)), dtype)
    kb.append_quantize(pool, seqs, 0, dev_bits(kd, dtype), dev_bits(vd, dtype))
    qb = to_bits(kv_values(rng, (layers, n, nq, hq, D)), dtype)
    out = torch.empty((layers, n, nq, hq, D), dtype=torch.float32, device="cuda")
    kb.verify_attention(pool, seqs, 0, dev_bits(qb, dtype), out, scale)
    torch.cuda.synchronize()
    assert pool.device_error() == 0
    # 9-16 columns per sequence (queries x GQA group) with 8+ kv heads run as
    # two 8-column query tiles of one decode item
    g = hq // hkv
    two_tiles = 8 < nq * g <= 16 and hkv >= 8 and D <= 128
    assert pool.last_kernels().split("+")[0].endswith(",2>") == two_tiles, pool.last_kernels()
    got = out.cpu().numpy().astype(np.float64)
    for i in range(n):
        for layer in range(layers):
            kk = np.concatenate([K[i][layer], kd[layer, i]], axis=1)
            vv = np.concatenate([V[i][layer], vd[layer, i]], axis=1)
            ck, sk, zk = oracle.quantize(kk, dtype, G)
            cv, sv, zv = oracle.quantize(vv, dtype, G)
            for j in range(nq):
                t = lengths[i] + j + 1  # the cache as the sequential step j sees it
                ref = oracle.reference_attention(ck[:, :t], sk[:, :t], zk[:, :t], cv[:, :t], sv[:, :t],
                                                 zv[:, :t], qb[layer, i, j], dtype, G, scale)
                err = np.abs(got[layer, i, j] - ref).max()
                assert err <= ATOL, f"seq {i} layer {layer} query {j}: {err:.3e}"
    pool.close()


@pytest.mark.parametrize("D,G,hq,hkv,dtype,prefix,chunk,impl", [
    (128, 64, 32, 8, BF16, 1000, 300, kb.ATTN_TENSOR_CORE),   # 1200 query rows: causal tcgen05 items
    (64, 64, 32, 8, F16, 77, 130, kb.ATTN_TENSOR_CORE),
    (128, 128, 16, 16, F16, 500, 64, kb.ATTN_TENSOR_CORE),    # MHA, G = D
    (128, 64, 32, 8, BF16, 1000, 300, kb.ATTN_TENSOR_CORE_PAIR),  # the same on CTA pairs
    (64, 64, 32, 8, F16, 77, 130, kb.ATTN_TENSOR_CORE_PAIR),
])
def test_prefill_attention_matches_oracle(D, G, hq, hkv, dtype, prefix, chunk, impl):
    """Chunked prefill (InferenceEngine.swift:3122-3147): append the chunk's
    K/V, then every chunk query attends the cache causally. Checked against
    the oracle at a spread of queries (first, last and every 13th)."""
    rng = np.random.default_rng(13)
    layers = 2
    scale = 1 / math.sqrt(D)
    pool = kb.KVPool(layers, hkv, hq, D, num_blocks=48, group_size=G, attn_impl=impl)
    seqs, K, V = [], [], []
    for L in (prefix, prefix // 3 + 1):
        s = pool.create_sequence()
        k = to_bits(kv_values(rng, (layers, hkv, L + chunk, D)), dtype)
        v = to_bits(kv_values(rng, (layers, hkv, L + chunk, D)), dtype)
        prefill(pool, s, k, v, dtype)  # prefix + this chunk
        seqs.append(s)
        K.append(k)
        V.append(v)
    n = len(seqs)
    qb = to_bits(kv_values(rng, (layers, n, chunk, hq, D)), dtype)
    out = torch.empty((layers, n, chunk, hq, D), dtype=torch.float32, device="cuda")
    kb.prefill_attention(pool, seqs, 0, dev_bits(qb, dtype), out, scale)
    torch.cuda.synchronize()
    assert pool.device_error() == 0
    assert ("attn_shared_pair_kernel" in pool.last_kernels()) == (
        impl == kb.ATTN_TENSOR_CORE_PAIR and chunk * (hq // hkv) > 128), pool.last_kernels()
    got = out.cpu().numpy().astype(np.float64)
    check_q = sorted(set(list(range(0, chunk, 13)) + [chunk - 1]))
    for i in range(n):
        total = K[i].shape[2]
        for layer in range(layers):
            ck, sk, zk = oracle.quantize(K[i][layer], dtype, G)
            cv, sv, zv = oracle.quantize(V[i][layer], dtype, G)
            for j in check_q:
                t = total - chunk + j + 1
                ref = oracle.reference_attention(ck[:, :t], sk[:, :t], zk[:, :t], cv[:, :t], sv[:, :t],
                                                 zv[:, :t], qb[layer, i, j], dtype, G, scale)
                err = np.abs(got[layer, i, j] - ref).max()
                assert err <= ATOL, f"seq {i} layer {layer} query {j}: {err:.3e}"
    pool.close()
