"""Cascade (shared-prefix) decode attention: requests forked from one
prefix-cache entry (PrefixCache.lookupQuantized + restore and truncate,
InferenceEngine.swift:1305-1320, 1378-1417) share the prefix's blocks, and
the shared part is attended by one cascade item per (layer, kv head, query
row block) that reads and dequantizes it once for all of them.

Each request's output must still match the reference math for that request
alone (its own full cache, fp16-dequantized, SDPA with GQA; float64 oracle),
within the decode-attention tolerance: max-abs 2e-3 on fp32 outputs, plus
one half-ulp of the output dtype for f16/bf16 outputs.
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
from tests.test_gpu_attention import ATOL, half_ulp  # noqa: E402


def run_cascade(D, G, hq, hkv, dtype, prefixes, scale, layers=2, extra=(), outliers=False,
                out_dtype=torch.float32, steps=2, seed=0, min_groups=1, min_slots=1,
                impl=kb.ATTN_TENSOR_CORE, expect_kernel=None):
    """prefixes: list of (prefix length, [suffix length per fork]). extra:
    lengths of independent sequences batched alongside. expect_kernel: a
    kernel name that the step's launch description must contain."""
    rng = np.random.default_rng(seed)
    total = sum(p + sum(s) + len(s) * 256 for p, s in prefixes) + sum(extra) + 1024
    pool = kb.KVPool(layers, hkv, hq, D, num_blocks=total // 256 + 16 * (len(extra) + 4),
                     group_size=G, attn_impl=impl)
    pc = kb.PrefixCache(pool)
    seqs, K, V = [], [], []
    for pi, (P, suffixes) in enumerate(prefixes):
        base = pool.create_sequence()
        kp = to_bits(kv_values(rng, (layers, hkv, P, D), outliers), dtype)
        vp = to_bits(kv_values(rng, (layers, hkv, P, D), outliers), dtype)
        prefill(pool, base, kp, vp, dtype)
        toks = [pi * 10_000_000 + t for t in range(P)]
        pc.store_quantized(toks, "m", base)
        base.release()
        hit = pc.lookup_quantized(toks, "m")
        for S in suffixes:
            f = hit.fork(P)
            kk, vv = kp, vp
            if S:
                ks = to_bits(kv_values(rng, (layers, hkv, S, D), outliers), dtype)
                vs = to_bits(kv_values(rng, (layers, hkv, S, D), outliers), dtype)
                prefill(pool, f, ks, vs, dtype)
                kk = np.concatenate([kp, ks], axis=2)
                vv = np.concatenate([vp, vs], axis=2)
            seqs.append(f)
            K.append(kk)
            V.append(vv)
        hit.release()
    for L in extra:
        s = pool.create_sequence()
        k = to_bits(kv_values(rng, (layers, hkv, L, D), outliers), dtype)
        v = to_bits(kv_values(rng, (layers, hkv, L, D), outliers), dtype)
        prefill(pool, s, k, v, dtype)
        seqs.append(s)
        K.append(k)
        V.append(v)
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
        groups, items, slots, ctas = pool.last_cascade()
        assert groups >= min_groups and items > 0 and slots >= min_slots and ctas > 0
        if expect_kernel is not None:
            assert expect_kernel in pool.last_kernels(), pool.last_kernels()
        assert pool.device_error() == 0
        got = out.float().cpu().numpy().astype(np.float64)
        for i in range(n):
            K[i] = np.concatenate([K[i], k1[:, i]], axis=2)
            V[i] = np.concatenate([V[i], v1[:, i]], axis=2)
            for layer in range(layers):
                ck, sk, zk = oracle.quantize(K[i][layer], dtype, G)
                cv, sv, zv = oracle.quantize(V[i][layer], dtype, G)
                ref = oracle.reference_attention(ck, sk, zk, cv, sv, zv, qb[layer, i], dtype, G, scale)
                err = np.abs(got[layer, i] - ref)
                tol = ATOL + half_ulp(ref, out_dtype)
                assert np.all(err <= tol), (
                    f"seq {i} (L={K[i].shape[2]}) layer {layer}: max err {err.max():.3e}")
                worst = max(worst, float(err.max()))
    pc.close()
    pool.close()
    return worst


@pytest.mark.parametrize("D,G,hq,hkv,dtype,scale", [
    (128, 64, 32, 8, BF16, 1 / math.sqrt(128)),  # Llama-3.1-8B shape (config 3)
    (64, 64, 32, 8, F16, 1 / 8),                  # D = 64, GQA 4
    (128, 64, 32, 4, BF16, 1 / math.sqrt(128)),   # GQA 8
    (256, 64, 8, 4, F16, 1.0),                    # D = 256 (16 rows per warp), GQA 2
    (128, 128, 16, 16, F16, 1 / math.sqrt(128)),  # G = D, MHA
    (256, 256, 16, 2, BF16, 1.0),                 # D = 256, G = D
])
def test_cascade_matches_oracle(D, G, hq, hkv, dtype, scale):
    run_cascade(D, G, hq, hkv, dtype, [(1024, [1, 17, 64, 100, 255, 300])], scale)


def test_cascade_fragments_and_empty_slots():
    # a 4096-token prefix over 4 layers is cut into fragments of unequal
    # count per (layer, head): several partial slots, some left empty
    run_cascade(128, 64, 32, 8, BF16, [(4096, [1, 70, 256, 300, 513])], 1 / math.sqrt(128),
                layers=4, steps=1, min_slots=2)


def test_cascade_row_blocks():
    # more members than one item's query rows: 70 forks x GQA 4 = 280 rows
    # (> 256 at D = 128), and 70 x GQA 2 = 140 rows (> 128 at D = 256)
    run_cascade(128, 64, 32, 8, BF16, [(512, [3 + (i % 7) for i in range(70)])],
                1 / math.sqrt(128), layers=1, steps=1)
    run_cascade(256, 64, 8, 4, F16, [(512, [3 + (i % 5) for i in range(70)])], 1.0, layers=1,
                steps=1)


def test_cascade_mixed_batch():
    # two prefix families, a fork with no suffix of its own (its decode items
    # cover only the appended token) and independent sequences, in one call
    run_cascade(128, 64, 32, 8, BF16, [(768, [0, 5, 129]), (1536, [40, 41])],
                1 / math.sqrt(128), extra=[9, 700], min_groups=2)


def test_cascade_outliers():
    # 1% N(0, 8) outliers: scales above 64 take the exact two-rounding dequant
    run_cascade(128, 64, 32, 4, BF16, [(1024, [10, 300])], 1 / math.sqrt(128), outliers=True,
                layers=1)


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.bfloat16])
def test_cascade_low_precision_out(out_dtype):
    run_cascade(128, 64, 32, 8, F16, [(512, [1, 2, 3])], 1 / math.sqrt(128), out_dtype=out_dtype,
                layers=1, steps=1)


@pytest.mark.parametrize("D,G,hq,hkv,dtype,scale", [
    (128, 64, 32, 8, BF16, 1 / math.sqrt(128)),
    (64, 64, 32, 8, F16, 1 / 8),
])
def test_cascade_mma_sync_variant(D, G, hq, hkv, dtype, scale):
    # the cascade part on mma.sync (KRILL_ATTN_TENSOR_CORE_SYNC), kept for comparison
    run_cascade(D, G, hq, hkv, dtype, [(1024, [1, 17, 64, 300])], scale,
                impl=kb.ATTN_TENSOR_CORE_SYNC)


PAIR = "attn_shared_pair_kernel"


@pytest.mark.parametrize("D,G,hq,hkv,dtype,scale,forks", [
    (128, 64, 32, 8, BF16, 1 / math.sqrt(128), 64),    # configs[2] shape: 256 rows per item
    (64, 64, 32, 8, F16, 1 / 8, 40),                   # D = 64: 160 rows
    (128, 64, 32, 4, BF16, 1 / math.sqrt(128), 20),    # GQA 8: 160 rows
    (128, 128, 16, 16, F16, 1 / math.sqrt(128), 150),  # G = D, MHA: items of 150 rows
])
def test_cascade_cta_pairs(D, G, hq, hkv, dtype, scale, forks):
    # KRILL_ATTN_TENSOR_CORE_PAIR: items of more than 128 query rows run on CTA
    # pairs (tcgen05 cta_group::2, M = 256 per instruction, each CTA
    # dequantizing half of every sub-block)
    run_cascade(D, G, hq, hkv, dtype, [(1024, [1 + (i * 37) % 300 for i in range(forks)])], scale,
                impl=kb.ATTN_TENSOR_CORE_PAIR, expect_kernel=PAIR)


def test_cascade_cta_pairs_outliers_fragments_and_rows():
    # scales above 64 (exact two-rounding dequant) on the pair kernel; a
    # 4096-token prefix over 4 layers cut into several fragments per (layer,
    # head); 70 forks x GQA 4 = 280 rows: one item of 256 rows and one of 24
    # (the second CTA of that pair has no rows of its own)
    pair = kb.ATTN_TENSOR_CORE_PAIR
    run_cascade(128, 64, 32, 4, BF16, [(1024, [10 + 3 * i for i in range(40)])], 1 / math.sqrt(128),
                outliers=True, layers=1, impl=pair, expect_kernel=PAIR)
    run_cascade(128, 64, 32, 8, BF16, [(4096, [1 + 5 * i for i in range(48)])], 1 / math.sqrt(128),
                layers=4, steps=1, min_slots=2, impl=pair, expect_kernel=PAIR)
    run_cascade(128, 64, 32, 8, BF16, [(512, [3 + (i % 7) for i in range(70)])], 1 / math.sqrt(128),
                layers=1, steps=1, impl=pair, expect_kernel=PAIR)


def test_cascade_single_cta_by_default():
    # the default tensor-core path keeps one CTA per item at any row count
    run_cascade(128, 64, 32, 8, BF16, [(1024, [1 + (i * 37) % 300 for i in range(64)])],
                1 / math.sqrt(128), layers=1, steps=1, expect_kernel="attn_shared_umma_kernel")
