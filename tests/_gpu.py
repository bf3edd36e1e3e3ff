"""GPU-test helpers: move seeded host data to the device and back. torch is
plumbing only (buffers, streams); every computation runs in libkrill_kv.so."""
import numpy as np
import torch

import krill_b200 as kb

TORCH16 = {0: torch.float16, 1: torch.bfloat16}


def dev_bits(bits: np.ndarray, dtype: int) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(TORCH16[dtype])
    return t.cuda()


def host_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def prefill(pool: kb.KVPool, seq, k_bits: np.ndarray, v_bits: np.ndarray, dtype: int, chunk: int = 0):
    """Append [layers, Hkv, L, D] K/V bits to one sequence (all layers)."""
    L = k_bits.shape[2]
    step = L if chunk <= 0 else chunk
    for t0 in range(0, L, step):
        t1 = min(L, t0 + step)
        k = dev_bits(np.ascontiguousarray(k_bits[:, None, :, t0:t1, :]), dtype)
        v = dev_bits(np.ascontiguousarray(v_bits[:, None, :, t0:t1, :]), dtype)
        kb.append_quantize(pool, [seq], 0, k, v)
