"""Pinning the CPU oracle (oracle/krill_oracle.cpp) before trusting it.

The reference (Swift + MLX, macOS only) cannot run here, so the oracle is
pinned against (1) the known answers and bounds in the reference's own tests,
(2) published FNV-1a test vectors, (3) an independent numpy restatement of
the quantizer written from QuantizedKVCache.swift:181-204, and (4) the
committed golden fixtures (tests/golden/, made by gen_golden.py).
"""
import os

import numpy as np
import pytest

import oracle
from tests._data import BF16, F16, kv_values, to_bits

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


# ----------------------------------------------------------- fp16 / bf16
def test_f16_conversion_matches_numpy_rn_even():
    rng = np.random.default_rng(0)
    x = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * 10,
        rng.standard_normal(2000).astype(np.float32) * 1e-5,   # subnormal range
        np.array([0.0, -0.0, 65504.0, 65519.9, 65520.0, 1e9, -1e9, 2.0 ** -24, 2.0 ** -25,
                  3 * 2.0 ** -25, 1.0 + 2.0 ** -11, 1.0 + 3 * 2.0 ** -11], np.float32),
    ])
    with np.errstate(over="ignore"):
        want = x.astype(np.float16).view(np.uint16)
    got = np.array([oracle.f32_to_f16_bits(v) for v in x], np.uint16)
    np.testing.assert_array_equal(got, want)


def test_bf16_conversion_rn_even_known_answers():
    cases = {1.0: 0x3F80, -2.0: 0xC000, 1.0 + 2.0 ** -8: 0x3F80,  # tie -> even
             1.0 + 3 * 2.0 ** -8: 0x3F82, 3.0: 0x4040, 65504.0: 0x4780}
    for v, bits in cases.items():
        assert oracle.f32_to_bf16_bits(v) == bits, v
    rng = np.random.default_rng(1)
    x = rng.standard_normal(5000).astype(np.float32)
    np.testing.assert_array_equal(to_bits(x, BF16),
                                  np.array([oracle.f32_to_bf16_bits(v) for v in x], np.uint16))


# ----------------------------------------------------------- quantizer
def _bf16_round(x32: np.ndarray) -> np.ndarray:
    return (to_bits(x32, BF16).astype(np.uint32) << 16).view(np.float32)


def numpy_quantize(bits: np.ndarray, dtype: int, G: int):
    """Independent restatement of QuantizedKVCache.quantizePerHead
    (QuantizedKVCache.swift:181-197) with numpy's IEEE float16/float32."""
    D = bits.shape[-1]
    if dtype == F16:
        x = bits.view(np.float16).reshape(-1, D // G, G)
        mn = x.min(axis=-1, keepdims=True)
        mx = x.max(axis=-1, keepdims=True)
        d = (mx - mn).astype(np.float16)                       # f16 subtract
        diff = (x - mn).astype(np.float16)                     # f16 subtract
        mn32 = mn.astype(np.float32)
    else:
        x = (bits.astype(np.uint32) << 16).view(np.float32).reshape(-1, D // G, G)
        mn = x.min(axis=-1, keepdims=True)
        mx = x.max(axis=-1, keepdims=True)
        d = _bf16_round(mx - mn)
        diff = _bf16_round(x - mn)
        mn32 = mn
    scale = np.maximum(d.astype(np.float32) / np.float32(255.0), np.float32(1e-8))
    n = diff.astype(np.float32) / scale
    n = np.minimum(np.maximum(n, np.float32(0)), np.float32(255))
    codes = n.astype(np.uint8).reshape(bits.shape)            # truncating cast
    s16 = scale.astype(np.float16).view(np.uint16).reshape(bits.shape[:-1] + (D // G,))
    z16 = mn32.astype(np.float16).view(np.uint16).reshape(bits.shape[:-1] + (D // G,))
    return codes, s16, z16


@pytest.mark.parametrize("dtype", [F16, BF16])
@pytest.mark.parametrize("D,G", [(64, 64), (128, 64), (128, 128), (256, 64)])
@pytest.mark.parametrize("outliers", [False, True])
def test_oracle_quantize_matches_numpy_restatement(dtype, D, G, outliers):
    rng = np.random.default_rng(D + G + dtype + 7 * outliers)
    bits = to_bits(kv_values(rng, (300, D), outliers), dtype)
    got = oracle.quantize(bits, dtype, G)
    want = numpy_quantize(bits, dtype, G)
    for a, b in zip(got, want):
        np.testing.assert_array_equal(a, b)


def test_quantize_known_answers():
    # constant row: d = 0 -> scale 1e-8 (stored as f16 0), codes 0, zero = x
    bits = to_bits(np.full((1, 64), 1.5, np.float32), F16)
    c, s, z = oracle.quantize(bits, F16, 64)
    assert (c == 0).all() and s[0, 0] == 0 and z[0, 0] == 0x3E00
    np.testing.assert_array_equal(oracle.dequantize(c, s, z, 64), bits)
    # ramp 0..63: scale = 63/255 in f32; the truncating cast gives 254 for the
    # max element when 63 / fl(63/255) rounds just below 255
    bits = to_bits(np.arange(64, dtype=np.float32)[None], F16)
    c, s, z = oracle.quantize(bits, F16, 64)
    scale = np.float32(63.0) / np.float32(255.0)
    want = np.floor(np.arange(64, dtype=np.float32) / scale).astype(np.uint8)
    np.testing.assert_array_equal(c[0], want)
    assert z[0, 0] == 0 and s[0, 0] == np.float16(scale).view(np.uint16)
    # min element always codes to 0, the max to 254 or 255
    rng = np.random.default_rng(3)
    bits = to_bits(rng.standard_normal((500, 64)).astype(np.float32), F16)
    c, _, _ = oracle.quantize(bits, F16, 64)
    assert (c.min(axis=1) == 0).all()
    assert np.isin(c.max(axis=1), [254, 255]).all()


def test_dequantize_two_fp16_roundings():
    rng = np.random.default_rng(4)
    bits = to_bits(rng.standard_normal((200, 128)).astype(np.float32), F16)
    c, s, z = oracle.quantize(bits, F16, 64)
    got = oracle.dequantize(c, s, z, 64).view(np.float16)
    sc = np.repeat(s.view(np.float16), 64, axis=1)
    zc = np.repeat(z.view(np.float16), 64, axis=1)
    want = (c.astype(np.float16) * sc).astype(np.float16) + zc      # QuantizedKVCache.swift:202-203
    np.testing.assert_array_equal(got.view(np.uint16), want.astype(np.float16).view(np.uint16))


def _weyl(lo, hi, shape=(1, 4, 8, 64)):
    total = int(np.prod(shape))
    span = np.float32(max(hi - lo, 1e-3))
    i = np.arange(total, dtype=np.float32)
    frac = i * np.float32(0.6180339887) - np.floor(i * np.float32(0.6180339887))
    return (np.float32(lo) + frac * span).reshape(shape)


@pytest.mark.parametrize("lo,hi,slack", [(0.0, 10.0, 1e-3), (0.0, 5.0, 1e-3), (-64.0, 64.0, 1e-2),
                                         (-32.0, 64.0, 1e-2), (-2.0, 2.0, 1e-3)])
def test_weyl_round_trip_bound(lo, hi, slack):
    """QuantizedKVCacheUnitTests.swift:38-84: round-trip error below
    1.5 * range / 255 + slack (head_dim 64 here; the reference test uses 16)."""
    bits = to_bits(_weyl(lo, hi), F16)
    c, s, z = oracle.quantize(bits, F16, 64)
    back = oracle.dequantize(c, s, z, 64).view(np.float16).astype(np.float32)
    err = np.abs(back - bits.view(np.float16).astype(np.float32)).max()
    assert err < (hi - lo) / 255.0 * 1.5 + slack


# ----------------------------------------------------------- SDPA
def test_sdpa_definition():
    rng = np.random.default_rng(5)
    q = rng.standard_normal((8, 64))
    k = rng.standard_normal((2, 50, 64))
    v = rng.standard_normal((2, 50, 64))
    got = oracle.sdpa_f64(q, k, v, 0.125)
    for h in range(8):
        kh = h // 4  # GQA: query head h reads kv head h / (Hq / Hkv)
        s = k[kh] @ q[h] * 0.125
        p = np.exp(s - s.max())
        np.testing.assert_allclose(got[h], p @ v[kh] / p.sum(), rtol=1e-12, atol=1e-12)
    # identical keys -> plain mean of the values
    k2 = np.ones((1, 7, 64))
    got = oracle.sdpa_f64(q[:1], k2, v[:1, :7], 1.0)
    np.testing.assert_allclose(got[0], v[0, :7].mean(axis=0), rtol=1e-12)


# ----------------------------------------------------------- prefix key
def test_fnv1a_published_vectors():
    assert oracle.fnv1a64(b"") == 0xCBF29CE484222325
    assert oracle.fnv1a64(b"a") == 0xAF63DC4C8601EC8C
    assert oracle.fnv1a64(b"foobar") == 0x85944171F73967E8


def test_prefix_key_layout():
    """PrefixCache.cacheKey (PrefixCache.swift:513-532): v3 || dtype || model
    || 0xFF || media (if non-empty) || 0xFF || Int64 LE tokens."""
    toks = [1, 2, 300000, -5]
    data = bytes([3, 2]) + b"m-int8" + b"\xff" + b"img" + b"\xff" + np.array(toks, "<i8").tobytes()
    assert oracle.prefix_key(toks, "m-int8", "img") == oracle.fnv1a64(data)
    data = bytes([3, 2]) + b"m" + b"\xff\xff" + np.array(toks, "<i8").tobytes()
    assert oracle.prefix_key(toks, "m", None) == oracle.fnv1a64(data)
    assert oracle.prefix_key(toks, "m", "") == oracle.fnv1a64(data)
    assert oracle.prefix_key(toks, "m", None, dtype_tag=1) != oracle.prefix_key(toks, "m", None)


# ----------------------------------------------------------- golden fixtures
def _fixtures(prefix):
    return sorted(f for f in os.listdir(GOLDEN) if f.startswith(prefix) and f.endswith(".npz"))


def test_golden_quantize_fixtures():
    files = _fixtures("quant_")
    assert files, "golden fixtures missing (run tests/golden/gen_golden.py)"
    for f in files:
        z = np.load(os.path.join(GOLDEN, f))
        c, s, zz = oracle.quantize(z["x"], int(z["dtype"]), int(z["G"]), int(z["variant"]))
        np.testing.assert_array_equal(c, z["codes"], err_msg=f)
        np.testing.assert_array_equal(s, z["scales"], err_msg=f)
        np.testing.assert_array_equal(zz, z["zeros"], err_msg=f)
        np.testing.assert_array_equal(oracle.dequantize(c, s, zz, int(z["G"])), z["deq"], err_msg=f)


def test_golden_attention_fixtures():
    files = _fixtures("attn_")
    assert files
    for f in files:
        z = np.load(os.path.join(GOLDEN, f))
        G = int(z["G"])
        dt = int(z["dtype"])
        ck, sk, zk = oracle.quantize(z["k"], dt, G)
        cv, sv, zv = oracle.quantize(z["v"], dt, G)
        out = oracle.reference_attention(ck, sk, zk, cv, sv, zv, z["q"], dt, G, float(z["scale"]))
        np.testing.assert_allclose(out, z["out"], rtol=0, atol=1e-12, err_msg=f)


def test_rope_restatement_against_float64():
    """The oracle's rotate-half RoPE (the rotation the reference applies to K
    before caching, traditional: false): identity at position 0, and within
    one rounding of the input dtype of the float64 rotation elsewhere."""
    rng = np.random.default_rng(11)
    D, rows = 128, 64
    cos, sin = oracle.rope_table(500000.0, D, rows)
    assert cos.dtype == np.float32 and cos.shape == (rows, D // 2)
    for dtype in (F16, BF16):
        x = to_bits(rng.standard_normal((3, 9, D)), dtype)
        pos = np.array([0, 1, 2, 5, 9, 17, 33, 40, 63])
        y = oracle.apply_rope(x, dtype, cos, sin, pos)
        np.testing.assert_array_equal(y[:, 0], x[:, 0])  # cos 1, sin 0
        xf = oracle.bits_to_f64(x, dtype)
        h = D // 2
        ang = pos[:, None] * (500000.0 ** (-2.0 * np.arange(h) / D))[None, :]
        c, s = np.cos(ang), np.sin(ang)
        ref = np.concatenate([xf[..., :h] * c - xf[..., h:] * s, xf[..., :h] * s + xf[..., h:] * c], -1)
        rel = 2.0 ** (-10 if dtype == F16 else -7)
        assert np.all(np.abs(oracle.bits_to_f64(y, dtype) - ref) <= rel * np.abs(ref) + 1e-6)


def _code_by_reciprocal(a, s):
    """numpy float32 restatement of the append kernels' quotient rule
    (code_of in kv_ops.cu): trunc(qa) for qa = RN(a * RN(1/s)) at least 1e-4
    from an integer k; else k or k - 1 by the sign of fma(-k, s, a) + h_k s
    (the exact test q >= k - h_k). fma(-k, s, a) is exact there; numpy
    evaluates it in float64, which is exact for these operands."""
    a = a.astype(np.float32)
    s = np.broadcast_to(s, a.shape).astype(np.float32)
    rinv = (np.float32(1.0) / s).astype(np.float32)
    qa = (a * rinv).astype(np.float32)
    k = np.rint(qa).astype(np.float32)
    far = np.abs(qa - k) >= np.float32(1e-4)
    r = (a.astype(np.float64) - k.astype(np.float64) * s.astype(np.float64)).astype(np.float32)
    km = (k - np.float32(0.5)).astype(np.float32)
    p2 = (km.view(np.uint32) & np.uint32(0x7F800000)).view(np.float32)
    up = (r + (s * np.float32(2.0 ** -24)).astype(np.float32) * p2).astype(np.float32)
    near_code = np.where(k >= 256, 255, np.where(k <= 0, 0, k.astype(np.int64) - (up < 0)))
    code = np.where(far, np.trunc(np.minimum(qa, 255)).astype(np.int64), near_code)
    return np.where(a == 0, 0, code).astype(np.uint8), ~far & (a != 0)


def test_quotient_by_reciprocal_matches_the_divide():
    """The append kernels compute trunc(clip(RN(a / s), 0, 255)) without a
    divide per element (code_of in kv_ops.cu). Check the rule against the
    IEEE divide on the quantizer's own operands: f16 and bf16 groups of 64
    (N(0,1), N(0,8), tiny and wide values, constant groups), a = rn_in(x - mn),
    s = max(RN(rn_in(mx - mn) / 255), 1e-8), float32 throughout
    (QuantizedKVCache.swift:185-194)."""
    rng = np.random.default_rng(123)
    checked = 0
    for dtype in (F16, BF16):
        for sigma in (1.0, 8.0, 1e-3, 300.0):
            x = rng.standard_normal((40000, 64)).astype(np.float32) * np.float32(sigma)
            x[:100] = x[:100, :1]  # constant groups
            xb = oracle.bits_to_f64(to_bits(x, dtype), dtype).astype(np.float32)

            def rn_in(v):
                return oracle.bits_to_f64(to_bits(v, dtype), dtype).astype(np.float32)

            mn = xb.min(axis=1, keepdims=True)
            d = rn_in(xb.max(axis=1, keepdims=True) - mn)
            s = np.maximum(d / np.float32(255.0), np.float32(1e-8)).astype(np.float32)
            a = rn_in(xb - mn)
            exact = np.trunc(np.clip(a / s, 0, 255)).astype(np.uint8)
            got, near = _code_by_reciprocal(a, s)
            assert np.array_equal(got, exact)
            if sigma >= 1.0:
                assert near.mean() < 0.05, near.mean()
            checked += a.size
    # every representable quotient near each integer boundary, both sides
    s = np.float32(1.0) / np.float32(255.0)
    for k in range(1, 257):
        q = np.float32(k) * s
        a = q + (np.arange(-20, 21, dtype=np.float32) * np.spacing(q))
        got, _ = _code_by_reciprocal(a.astype(np.float32), s)
        assert np.array_equal(got, np.trunc(np.clip(a / s, 0, 255)).astype(np.uint8))
    assert checked > 10_000_000
