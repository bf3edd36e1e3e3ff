#!/usr/bin/env python3
"""Generates the golden fixtures in this directory from seeded inputs with the
CPU oracle (oracle/krill_oracle.cpp).

The reference (Swift + MLX, macOS only) cannot run on this platform, so these
vectors freeze the oracle restatement (itself checked against the
reference's known answers and an independent numpy restatement in
tests/test_oracle.py). They pin the CUDA kernels: tests/test_gpu_golden.py
feeds the same inputs through the C ABI and requires bit-exact codes, scales,
zeros and dequantized values, and attention within 2e-3.

Run from the repository root:  python tests/golden/gen_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from tests._data import BF16, F16, kv_values, to_bits  # noqa: E402

QUANT_CASES = [
    # name, rows, D, G, dtype, variant, outliers
    ("quant_d64_f16", 96, 64, 64, F16, 0, False),
    ("quant_d128_g64_bf16", 96, 128, 64, BF16, 0, False),
    ("quant_d128_g64_bf16_outliers", 96, 128, 64, BF16, 0, True),
    ("quant_d128_g128_f16", 96, 128, 128, F16, 0, False),
    ("quant_d256_g64_f16", 64, 256, 64, F16, 0, True),
    ("quant_d128_g64_f16_inputdtype", 96, 128, 64, F16, 1, False),
]

ATTN_CASES = [
    # name, D, G, Hq, Hkv, L, dtype, scale
    ("attn_d64_l70_f16", 64, 64, 32, 8, 70, F16, 1 / 8.0),
    ("attn_d128_l300_bf16", 128, 64, 32, 8, 300, BF16, 1 / np.sqrt(128.0)),
    ("attn_d128_gqa8_l129_bf16", 128, 64, 32, 4, 129, BF16, 1 / np.sqrt(128.0)),
    ("attn_d256_l65_f16", 256, 64, 8, 4, 65, F16, 1.0),
]


def main():
    for i, (name, rows, D, G, dt, var, outl) in enumerate(QUANT_CASES):
        rng = np.random.default_rng(100 + i)
        x = to_bits(kv_values(rng, (rows, D), outl), dt)
        c, s, z = oracle.quantize(x, dt, G, var)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), x=x, dtype=dt, G=G, variant=var,
                            codes=c, scales=s, zeros=z, deq=oracle.dequantize(c, s, z, G))
    for i, (name, D, G, hq, hkv, L, dt, scale) in enumerate(ATTN_CASES):
        rng = np.random.default_rng(200 + i)
        k = to_bits(kv_values(rng, (hkv, L, D)), dt)
        v = to_bits(kv_values(rng, (hkv, L, D)), dt)
        q = to_bits(kv_values(rng, (hq, D)), dt)
        ck, sk, zk = oracle.quantize(k, dt, G)
        cv, sv, zv = oracle.quantize(v, dt, G)
        out = oracle.reference_attention(ck, sk, zk, cv, sv, zv, q, dt, G, scale)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), k=k, v=v, q=q, dtype=dt, G=G,
                            hq=hq, hkv=hkv, scale=scale, out=out)
    print("wrote", len(QUANT_CASES) + len(ATTN_CASES), "fixtures to", HERE)


if __name__ == "__main__":
    main()
