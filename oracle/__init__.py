"""ctypes wrapper of the CPU oracle (libkrill_oracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline arm, always as the checker or the reported CPU
baseline — never by the product (krill_b200/). See krill_oracle.cpp for the
restated reference functions and the pinning status (partially pinned; SDPA
values unpinned).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libkrill_oracle.so")


def build():
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


if not os.path.exists(LIB_PATH):
    build()

_lib = C.CDLL(LIB_PATH)
_p = C.c_void_p
_lib.oracle_quantize.argtypes = [_p, C.c_int, C.c_int64, C.c_int, C.c_int, C.c_int, _p, _p, _p]
_lib.oracle_dequantize.argtypes = [_p, _p, _p, C.c_int64, C.c_int, C.c_int, _p]
_lib.oracle_sdpa_f64.argtypes = [_p, _p, _p, C.c_int, C.c_int, C.c_int64, C.c_int, C.c_double, _p]
_lib.oracle_fnv1a64.argtypes = [_p, C.c_int64]
_lib.oracle_fnv1a64.restype = C.c_uint64
_lib.oracle_prefix_key.argtypes = [_p, C.c_int64, C.c_char_p, C.c_char_p, C.c_int]
_lib.oracle_prefix_key.restype = C.c_uint64
_lib.oracle_f32_to_f16.argtypes = [C.c_float]
_lib.oracle_f32_to_f16.restype = C.c_uint16
_lib.oracle_f32_to_bf16.argtypes = [C.c_float]
_lib.oracle_f32_to_bf16.restype = C.c_uint16
_lib.oracle_f16_to_f32.argtypes = [C.c_uint16]
_lib.oracle_f16_to_f32.restype = C.c_float
_lib.oracle_bf16_to_f32.argtypes = [C.c_uint16]
_lib.oracle_bf16_to_f32.restype = C.c_float
_lib.oracle_baseline_create.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int64, C.c_int64, C.c_uint64]
_lib.oracle_baseline_create.restype = _p
_lib.oracle_baseline_destroy.argtypes = [_p]
_lib.oracle_baseline_step.argtypes = [_p, C.c_int64, _p, _p, _p, C.c_int, C.c_int, C.c_float, _p, C.c_int]
_lib.oracle_hardware_concurrency.restype = C.c_int

F16, BF16 = 0, 1


def _ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_p)


def quantize(x_bits: np.ndarray, dtype: int, group: int, variant: int = 0):
    """x_bits: uint16 array [..., D] of f16 (dtype 0) or bf16 (dtype 1) bits.
    Returns (codes u8 [..., D], scales f16-bits [..., D/G], zeros f16-bits)."""
    x = np.ascontiguousarray(x_bits, dtype=np.uint16)
    D = x.shape[-1]
    rows = x.size // D
    ng = D // group
    codes = np.empty(x.shape, np.uint8)
    scales = np.empty(x.shape[:-1] + (ng,), np.uint16)
    zeros = np.empty_like(scales)
    _lib.oracle_quantize(_ptr(x), dtype, rows, D, group, variant, _ptr(codes), _ptr(scales), _ptr(zeros))
    return codes, scales, zeros


def dequantize(codes: np.ndarray, scales: np.ndarray, zeros: np.ndarray, group: int) -> np.ndarray:
    """Reference dequantize -> f16 bits, same shape as codes."""
    c = np.ascontiguousarray(codes, np.uint8)
    s = np.ascontiguousarray(scales, np.uint16)
    z = np.ascontiguousarray(zeros, np.uint16)
    D = c.shape[-1]
    out = np.empty(c.shape, np.uint16)
    _lib.oracle_dequantize(_ptr(c), _ptr(s), _ptr(z), c.size // D, D, group, _ptr(out))
    return out


def sdpa_f64(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float) -> np.ndarray:
    """q [Hq, D], k/v [Hkv, L, D] (float64) -> out [Hq, D] float64."""
    q = np.ascontiguousarray(q, np.float64)
    k = np.ascontiguousarray(k, np.float64)
    v = np.ascontiguousarray(v, np.float64)
    Hq, D = q.shape
    Hkv, L, _ = k.shape
    out = np.empty((Hq, D), np.float64)
    _lib.oracle_sdpa_f64(_ptr(q), _ptr(k), _ptr(v), Hq, Hkv, L, D, float(scale), _ptr(out))
    return out


def rope_table(base: float, head_dim: int, rows: int):
    """cos / sin [rows][head_dim/2] float32 of angle(p, d) = p * base^(-2d/head_dim),
    evaluated in float64 (the rotary frequencies of MLXFast.RoPE with
    traditional: false, as set up at Sources/KrillCore/Attention.swift:55)."""
    half = head_dim // 2
    inv = base ** (-2.0 * np.arange(half, dtype=np.float64) / head_dim)
    ang = np.arange(rows, dtype=np.float64)[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def apply_rope(x_bits: np.ndarray, dtype: int, cos: np.ndarray, sin: np.ndarray,
               positions: np.ndarray) -> np.ndarray:
    """Rotate-half RoPE of [..., T, D] bits at `positions` [T]: element d <
    D/2 -> x[d] c - x[d+h] s, element d + h -> x[d] s + x[d+h] c, every
    product and sum in float32, the result rounded to `dtype` (the rotated K
    the reference quantizes, Gemma4Model.swift:502-509). Returns bits."""
    x = bits_to_f64(x_bits, dtype).astype(np.float32)
    h = x.shape[-1] // 2
    c = cos[positions]
    s = sin[positions]
    x1, x2 = x[..., :h], x[..., h:]
    y1 = (x1 * c).astype(np.float32) - (x2 * s).astype(np.float32)
    y2 = (x1 * s).astype(np.float32) + (x2 * c).astype(np.float32)
    y = np.concatenate([y1, y2], axis=-1).astype(np.float32)
    if dtype == 0:
        return y.astype(np.float16).view(np.uint16)
    u = y.view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def f16_bits_to_f64(b: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(b, np.uint16).view(np.float16).astype(np.float64)


def bf16_bits_to_f64(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def bits_to_f64(b: np.ndarray, dtype: int) -> np.ndarray:
    return f16_bits_to_f64(b) if dtype == F16 else bf16_bits_to_f64(b)


def f32_to_f16_bits(x: float) -> int:
    return int(_lib.oracle_f32_to_f16(float(x)))


def f32_to_bf16_bits(x: float) -> int:
    return int(_lib.oracle_f32_to_bf16(float(x)))


def fnv1a64(data: bytes) -> int:
    buf = (C.c_uint8 * max(1, len(data))).from_buffer_copy(data or b"\0")
    return int(_lib.oracle_fnv1a64(buf, len(data)))


def prefix_key(tokens, model_id: str, media_hash=None, dtype_tag: int = 2) -> int:
    arr = np.ascontiguousarray(np.asarray(tokens, dtype=np.int64))
    return int(_lib.oracle_prefix_key(_ptr(arr) if arr.size else None, arr.size,
                                      model_id.encode(), None if media_hash is None else media_hash.encode(),
                                      dtype_tag))


def reference_attention(codes_k, sk, zk, codes_v, sv, zv, q_bits, q_dtype, group, scale):
    """Reference decode attention for one (sequence, layer): the reference
    dequantizes the whole cache to f16 (QuantizedKVCache.swift:72-73) and runs
    SDPA; here SDPA is evaluated in float64. codes [Hkv, L, D]; meta
    [Hkv, L, D/G]; q_bits [Hq, D] (f16/bf16 bits). Returns [Hq, D] float64."""
    kd = f16_bits_to_f64(dequantize(codes_k, sk, zk, group))
    vd = f16_bits_to_f64(dequantize(codes_v, sv, zv, group))
    return sdpa_f64(bits_to_f64(q_bits, q_dtype), kd, vd, scale)


def hardware_concurrency() -> int:
    return int(_lib.oracle_hardware_concurrency())


class Baseline:
    """CPU restatement of the reference's per-step dataflow (quantize, concat
    copy, full dequant, f32 SDPA) over n caches; see krill_oracle.cpp."""

    def __init__(self, n: int, Hkv: int, D: int, G: int, lengths, steps: int, seed: int = 0):
        self.caches = [_lib.oracle_baseline_create(Hkv, D, G, int(L), int(L) + steps + 1, seed + i)
                       for i, L in enumerate(lengths)]
        assert len(self.caches) == n
        self.arr = (C.c_void_p * n)(*self.caches)
        self.n = n

    def step(self, knew, vnew, q, Hq, dtype, scale, out, threads):
        _lib.oracle_baseline_step(self.arr, self.n, _ptr(knew), _ptr(vnew), _ptr(q), Hq, dtype,
                                  float(scale), _ptr(out), threads)

    def close(self):
        for c in self.caches:
            _lib.oracle_baseline_destroy(c)
        self.caches = []
