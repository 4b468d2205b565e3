"""Expert placement for expert parallelism.

Every rank holds the same number of experts (E / nranks).  With a skewed
expert popularity (the Zipf-routed prefill workload), contiguous id ranges put
the hot experts together; ``balanced_owner`` instead assigns experts greedily
by expected load (longest-processing-time first) under the equal-count
constraint, so each rank receives a similar number of routes.
"""
from __future__ import annotations

import numpy as np


def contiguous_owner(num_experts: int, nranks: int) -> np.ndarray:
    if num_experts % nranks:
        raise ValueError("experts must divide evenly over ranks")
    per = num_experts // nranks
    return (np.arange(num_experts) // per).astype(np.int32)


def balanced_owner(load, nranks: int) -> np.ndarray:
    load = np.asarray(load, np.float64)
    E = load.size
    if E % nranks:
        raise ValueError("experts must divide evenly over ranks")
    per = E // nranks
    owner = np.empty(E, np.int32)
    total = np.zeros(nranks)
    count = np.zeros(nranks, np.int64)
    for e in np.argsort(-load, kind="stable"):
        free = np.flatnonzero(count < per)
        r = free[np.argmin(total[free])]
        owner[e] = r
        total[r] += load[e]
        count[r] += 1
    return owner


def local_experts(owner, rank: int) -> np.ndarray:
    """Global ids held by ``rank``, ascending (the packing order of ep_set_layer)."""
    return np.flatnonzero(np.asarray(owner) == rank)
