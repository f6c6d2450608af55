"""
Neighbour lists in numpy: the bit-exact oracle of cg_neighbor_list.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py). The reference has no
neighbour list (models build theirs before the region, README.md:28 there),
so parity is anchored on this restatement of the stated rule: within each
system, the other atoms with d2 < cutoff^2, d2 = (dx*dx + dy*dy) + dz*dz in
float32 round-to-nearest operations (numpy's float32 arithmetic performs each
operation separately, so no fused multiply-add), the k nearest by (d2, j).
"""

from __future__ import annotations

import numpy as np


def neighbor_list(pos: np.ndarray, sys_ptr: np.ndarray, cutoff: float, k: int):
    """(nbr (n, k) int32 padded with -1, counts (n,), rev_ptr (n+1,), rev_idx)."""
    pos = np.asarray(pos, dtype=np.float32)
    n = pos.shape[0]
    cut2 = np.float32(cutoff) * np.float32(cutoff)
    nbr = np.full((n, k), -1, dtype=np.int32)
    counts = np.zeros(n, dtype=np.int32)
    for b in range(len(sys_ptr) - 1):
        a0, a1 = int(sys_ptr[b]), int(sys_ptr[b + 1])
        p = pos[a0:a1]
        d = p[None, :, :] - p[:, None, :]  # d[i, j] = pos[j] - pos[i], float32
        d2 = (d[..., 0] * d[..., 0] + d[..., 1] * d[..., 1]) + d[..., 2] * d[..., 2]
        for i in range(a1 - a0):
            js = np.array([j for j in range(a1 - a0) if j != i and d2[i, j] < cut2], dtype=np.int64)
            if js.size:
                order = np.lexsort((js, d2[i, js]))[:k]  # by d2, then index
                keep = js[order] + a0
                nbr[a0 + i, : keep.size] = keep
                counts[a0 + i] = keep.size
    slots = np.flatnonzero(nbr.reshape(-1) >= 0)
    targets = nbr.reshape(-1)[slots]
    order = np.lexsort((slots, targets))
    rev_idx = slots[order].astype(np.int32)
    rev_ptr = np.zeros(n + 1, dtype=np.int32)
    rev_ptr[1:] = np.cumsum(np.bincount(targets, minlength=n))
    return nbr, counts, rev_ptr, rev_idx
