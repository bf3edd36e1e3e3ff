"""Seeded synthetic inputs shared by the tests (no dataset is involved)."""
import numpy as np

F16, BF16 = 0, 1


def to_bits(x: np.ndarray, dtype: int) -> np.ndarray:
    """float array -> uint16 bits of f16 (RN) or bf16 (RN-even)."""
    if dtype == F16:
        return np.ascontiguousarray(x, np.float32).astype(np.float16).view(np.uint16)
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def kv_values(rng: np.random.Generator, shape, outliers: bool = False) -> np.ndarray:
    """N(0,1) values, or N(0, 0.5) with 1% outliers ~ N(0, 8)."""
    if not outliers:
        return rng.standard_normal(shape, dtype=np.float32)
    x = rng.standard_normal(shape, dtype=np.float32) * np.float32(np.sqrt(0.5))
    mask = rng.random(shape) < 0.01
    x[mask] = rng.standard_normal(int(mask.sum()), dtype=np.float32) * np.float32(np.sqrt(8.0))
    return x
