"""Sequence sharding across the GPUs of one node.

Decode attention and append never mix sequences, so the path shards by whole
sequences: one process per GPU, each with its own pool, no collective on the
data path. Sequences are assigned by longest-processing-time on their
expected bytes (sum over layers of the attended length); a prefix entry owned
by another GPU is fetched once with krill_prefix_peer_fetch.
"""
from __future__ import annotations

from typing import List, Sequence


def lpt_partition(weights: Sequence[int], n_parts: int) -> List[List[int]]:
    """Indices of `weights` split into n_parts lists, longest first onto the
    least-loaded part (ties: lowest index). Each part is returned sorted."""
    if n_parts <= 0:
        raise ValueError("n_parts must be positive")
    order = sorted(range(len(weights)), key=lambda i: (-weights[i], i))
    loads = [0] * n_parts
    parts: List[List[int]] = [[] for _ in range(n_parts)]
    for i in order:
        r = min(range(n_parts), key=lambda j: (loads[j], j))
        parts[r].append(i)
        loads[r] += weights[i]
    return [sorted(p) for p in parts]


def sequence_weight(length: int, num_layers: int, window: int = 0) -> int:
    """Attended tokens summed over layers (sliding layers see min(L, window))."""
    return num_layers * (min(length, window) if window > 0 else length)
